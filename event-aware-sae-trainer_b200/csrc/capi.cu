// C-ABI entry points of libsae_b200.so: argument checks, workspace carving,
// TMA descriptor set-up and the launch sequence of each step phase.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "dense_kernels.cuh"
#include "sae_b200.h"
#include "step_kernels.cuh"
#include "aux_kernels.cuh"
#include "peer_kernels.cuh"
#include "tile_gemm.cuh"
#include "gemm_kernels.cuh"

#include <type_traits>

using namespace sae;

namespace {

thread_local std::string g_last_error;
std::atomic<int64_t> g_launches{0};
constexpr int kTimers = 6;
cudaEvent_t g_timer_start[kTimers] = {};
cudaEvent_t g_timer_stop[kTimers] = {};

void timer_begin(int which, cudaStream_t s) {
  if (g_timer_start[which] != nullptr) cudaEventRecord(g_timer_start[which], s);
}
void timer_end(int which, cudaStream_t s) {
  if (g_timer_stop[which] != nullptr) cudaEventRecord(g_timer_stop[which], s);
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SAE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return SAE_OK;
}

#define SAE_TRY(expr)            \
  do {                           \
    const int _rc = (expr);      \
    if (_rc != SAE_OK) return _rc; \
  } while (0)

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct DeviceInfo {
  int sm_count = 0;
  int major = 0;
};

constexpr int kMaxDevices = 64;
constexpr int kMaxGridY = 65535;   // CUDA's limit on gridDim.y

DeviceInfo device_info() {
  static std::mutex mu;
  static DeviceInfo cache[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && cache[dev].sm_count == 0) {
    cudaDeviceGetAttribute(&cache[dev].sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
  }
  return (dev >= 0 && dev < 64) ? cache[dev] : DeviceInfo{};
}

// ------------------------------------------------------------ workspace
struct Layout {
  size_t theta, xc, pre, sbits, mask, tile_cnt, col_tot, col_act, col_offs, go, tok_sqerr,
      tok_cnt, gosum_part, thr_part, dbenc_part, db_enc, gemv_part, csr_tok, csr_val, sumsq_part,
      row_sumsq, order_k0, order_k1, order_v0, order_v1, order_tmp, order_tmp_bytes, counters,
      cut, total;
};

// Row pitch (tokens) of the feature-major pre-activations: whole 64-token
// boxes plus one, so that the pitch is never a power of two (a 2^k-byte pitch
// puts the 128 rows of every TMA box on the same DRAM channels).
inline int64_t pre_pitch(int64_t B) {
  int64_t p = (B + 63) / 64 * 64 + 64;
  if ((p & (p - 1)) == 0) p += 64;
  return p;
}

// Bits of a per-token active count (at most F).
int count_key_bits(int64_t F) {
  int b = 1;
  while ((int64_t(1) << b) <= F) ++b;
  return b;
}

Layout make_layout(int64_t B, int64_t d, int64_t F, int64_t cap) {
  Layout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t W = static_cast<size_t>((F + 31) / 32);
  // per-feature counts and partial sums per 128-token half of each token tile
  const size_t nT = 2 * static_cast<size_t>((B + TILE_N - 1) / TILE_N);
  L.theta = take(F * 4);
  L.xc = take(B * d * 2);
  L.pre = take(static_cast<size_t>(F) * pre_pitch(B) * 2);   // feature-major [F, ldp]
  L.sbits = take(static_cast<size_t>(F) * (pre_pitch(B) / 32) * 4);
  L.mask = take(B * W * 4);
  L.tile_cnt = take(nT * F * 4);
  // per-feature totals, adjacent (one memset): col_tot [F + 1] (entry
  // counts, then a 0 so that the exclusive scan of F + 1 ends in the total),
  // col_act [F] (active counts)
  L.col_tot = take((2 * F + 1) * 4);
  L.col_act = L.col_tot + (F + 1) * 4;
  L.col_offs = take((F + 1) * 4);
  L.go = take(B * d * 2);
  L.tok_sqerr = take(B * 4);
  L.tok_cnt = take(B * 4);
  L.gosum_part = take(static_cast<size_t>(DECODE_GRID) * d * 4);
  L.thr_part = take(nT * F * 4);
  L.dbenc_part = take(nT * F * 4);
  L.db_enc = take(F * 4);
  L.gemv_part = take(static_cast<size_t>(GEMV_GRID) * d * 4);
  L.csr_tok = take(cap * 4);
  L.csr_val = take(cap * 4);
  L.sumsq_part = take(NORM_GRID * 4);
  // per-(feature, warp) sums of squares of the final W_enc / W_dec / b_enc /
  // log_threshold gradients, written by the sampled backward (<= 32 warps)
  L.row_sumsq = take(static_cast<size_t>(F) * 32 * 4);
  // decode order: tokens sorted by active count, heaviest first
  L.order_k0 = take(B * 4);
  L.order_k1 = take(B * 4);
  L.order_v0 = take(B * 4);
  L.order_v1 = take(B * 4);
  size_t sort_bytes = 0;
  cub::DeviceRadixSort::SortPairsDescending(nullptr, sort_bytes, static_cast<int*>(nullptr),
                                            static_cast<int*>(nullptr),
                                            static_cast<int*>(nullptr),
                                            static_cast<int*>(nullptr), static_cast<int>(B), 0,
                                            count_key_bits(F));
  size_t scan_bytes = 0;   // the same scratch serves the CSR offset scan
  cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<int*>(nullptr),
                                static_cast<int*>(nullptr), static_cast<int>(F + 1));
  L.order_tmp_bytes = std::max(sort_bytes, scan_bytes);
  L.order_tmp = take(L.order_tmp_bytes);
  L.counters = take(256);
  L.cut = take(F * 8);   // per-feature gate cut values (float2)
  L.total = off;
  return L;
}

struct Ws {
  float* theta;
  bf16* xc;
  bf16* pre;
  uint32_t* sbits;
  uint32_t* mask;
  int* tile_cnt;
  int* col_tot;
  int* col_act;
  int* col_offs;
  bf16* go;
  float* tok_sqerr;
  int* tok_cnt;
  float* gosum_part;
  float* thr_part;
  float* dbenc_part;
  float* db_enc;
  float* gemv_part;
  int* csr_tok;
  uint32_t* csr_val;
  float* sumsq_part;
  float* row_sumsq;
  int *order_k0, *order_k1, *order_v0, *order_v1;
  void* order_tmp;
  size_t order_tmp_bytes;
  int* counters;
  float2* cut;
};

Ws carve(void* base, const Layout& L) {
  auto at = [&](size_t o) { return static_cast<uint8_t*>(base) + o; };
  Ws w;
  w.theta = reinterpret_cast<float*>(at(L.theta));
  w.xc = reinterpret_cast<bf16*>(at(L.xc));
  w.pre = reinterpret_cast<bf16*>(at(L.pre));
  w.sbits = reinterpret_cast<uint32_t*>(at(L.sbits));
  w.mask = reinterpret_cast<uint32_t*>(at(L.mask));
  w.tile_cnt = reinterpret_cast<int*>(at(L.tile_cnt));
  w.col_tot = reinterpret_cast<int*>(at(L.col_tot));
  w.col_act = reinterpret_cast<int*>(at(L.col_act));
  w.col_offs = reinterpret_cast<int*>(at(L.col_offs));
  w.go = reinterpret_cast<bf16*>(at(L.go));
  w.tok_sqerr = reinterpret_cast<float*>(at(L.tok_sqerr));
  w.tok_cnt = reinterpret_cast<int*>(at(L.tok_cnt));
  w.gosum_part = reinterpret_cast<float*>(at(L.gosum_part));
  w.thr_part = reinterpret_cast<float*>(at(L.thr_part));
  w.dbenc_part = reinterpret_cast<float*>(at(L.dbenc_part));
  w.db_enc = reinterpret_cast<float*>(at(L.db_enc));
  w.gemv_part = reinterpret_cast<float*>(at(L.gemv_part));
  w.csr_tok = reinterpret_cast<int*>(at(L.csr_tok));
  w.csr_val = reinterpret_cast<uint32_t*>(at(L.csr_val));
  w.sumsq_part = reinterpret_cast<float*>(at(L.sumsq_part));
  w.row_sumsq = reinterpret_cast<float*>(at(L.row_sumsq));
  w.order_k0 = reinterpret_cast<int*>(at(L.order_k0));
  w.order_k1 = reinterpret_cast<int*>(at(L.order_k1));
  w.order_v0 = reinterpret_cast<int*>(at(L.order_v0));
  w.order_v1 = reinterpret_cast<int*>(at(L.order_v1));
  w.order_tmp = at(L.order_tmp);
  w.order_tmp_bytes = L.order_tmp_bytes;
  w.counters = reinterpret_cast<int*>(at(L.counters));
  w.cut = reinterpret_cast<float2*>(at(L.cut));
  return w;
}

// ------------------------------------------------------------------ TMA
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Row-major bf16 [rows, cols] matrix in boxes of box_rows x box_cols.
int make_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
              uint32_t box_cols = TILE_K,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B, uint64_t pitch = 0) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr) return fail(SAE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (pitch == 0) pitch = cols;
  if (!aligned16(base) || (pitch * 2) % 16 != 0)
    return fail(SAE_ERR_MISALIGNED, "TMA operand must be 16-byte aligned with 16-byte row pitch");
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {pitch * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r =
      fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride, box,
         estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SAE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return SAE_OK;
}

// SAE_B200_PAIR=0 keeps the tile GEMMs on single CTAs (tcgen05 cta_group::1).
bool pair_mode_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SAE_B200_PAIR");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

// Feature tiles (pairs) per rasterisation group of the tile GEMMs;
// SAE_B200_GROUP_M overrides the default (1..1024).
int raster_group() {
  static const int g = [] {
    const char* v = std::getenv("SAE_B200_GROUP_M");
    const int x = v != nullptr ? std::atoi(v) : TC_GROUP_M;
    return std::max(1, std::min(1024, x));
  }();
  return g;
}

bool tc_eligible(int64_t d, int64_t F, int force_simt) {
  if (force_simt) return false;
  const DeviceInfo di = device_info();
  return di.major == 10 && d % TILE_K == 0 && F % TILE_M == 0 && d <= 65536;
}

// The sampled backward over a feature-major CSR: one feature (segment) per
// block of d / (8 U) threads (U = 2 for wide rows: more features in flight
// per SM). seg_rows maps segments to feature rows (the aux backward).
// Threads per block of the sampled backward at row width d (a multiple of 32).
// 16-byte column vectors per thread (U) of the sampled backward. Fewer warps
// per feature row mean less per-warp work per entry (the butterfly, the
// partial sums, the flag logic): at d = 1536, U = 3 (2 warps) measured
// 1.36 ms per 32768-token step against 1.51 ms for U = 2 (3 warps) and
// 2.0-2.1 ms for U = 1 (6 warps). U = 3 where the row splits into whole warps
// of 3 vectors, else 2 from d = 1024 up, else 1. SAE_B200_SAMPLED_U=1|2|3
// overrides it.
int sampled_u(int d) {
  static const int forced = [] {
    const char* v = std::getenv("SAE_B200_SAMPLED_U");
    return v != nullptr ? std::atoi(v) : 0;
  }();
  const int nvec = d / 8;
  if ((forced == 1 || forced == 2 || forced == 3) && nvec % forced == 0) return forced;
  if (nvec % 3 == 0 && (nvec / 3) % 32 == 0 && nvec / 3 >= 64) return 3;
  return (nvec % 2 == 0 && nvec / 2 >= 64) ? 2 : 1;
}


int sampled_threads(int d) {
  return (d / 8 / sampled_u(d) + 31) / 32 * 32;
}

void launch_sampled(const int* offs, const int* tok, const uint32_t* val, const bf16* go,
                    const bf16* xc, const bf16* w_dec, const float* theta, int n_seg,
                    int n_tokens, int d, float eps, int accumulate, float* g_wdec, float* g_wenc,
                    float* g_logthr, float* g_benc, float* db_enc, int* counter,
                    const SaeB200StepStats* stats, const int* seg_rows, int honor_overflow,
                    cudaStream_t stream, float* row_sumsq = nullptr) {
  const int U = sampled_u(d);
  const int bthr = sampled_threads(d);
  // blocks per SM the launch bounds allow: at 2 warps per block (U = 3), 8
  // blocks cap the registers at 128 (each SM sub-partition's 16K registers
  // hold 4 warps) without spills, measured 1.21 ms per 32768-token step
  // against 1.24 ms at 6 blocks; at 3 warps (U = 2) 6 blocks measured slower
  // than 5 (1.62 / 1.51 ms)
  const int per_sm = bthr <= 64 ? 8 : bthr <= 96 ? 5 : (bthr <= 192 ? 4 : (bthr <= 256 ? 2 : 1));
  const int grid = device_info().sm_count * per_sm * 2;
#define SAE_SAMPLED(CC, UU, MT, MB)                                                            \
  sampled_backward_kernel<CC, UU, MT, MB><<<grid, bthr, 0, stream>>>(                         \
      offs, tok, val, go, xc, w_dec, theta, n_seg, n_tokens, d, eps, accumulate, g_wdec,       \
      g_wenc, g_logthr, g_benc, db_enc, counter, stats, seg_rows, honor_overflow, row_sumsq)
  if (U == 3) {
    if (bthr <= 64) SAE_SAMPLED(2, 3, 64, 8);
    else SAE_SAMPLED(2, 3, 192, 2);
  } else if (U == 1) {
    if (bthr <= 192) SAE_SAMPLED(2, 1, 192, 4);
    else if (bthr <= 256) SAE_SAMPLED(4, 1, 256, 2);
    else if (bthr <= 512) SAE_SAMPLED(4, 1, 512, 1);
    else SAE_SAMPLED(4, 1, 1024, 1);
  } else {
    if (bthr <= 96) SAE_SAMPLED(2, 2, 96, 5);
    else if (bthr <= 192) SAE_SAMPLED(2, 2, 192, 2);
    else if (bthr <= 256) SAE_SAMPLED(2, 2, 256, 2);
    else SAE_SAMPLED(2, 2, 512, 1);
  }
#undef SAE_SAMPLED
}

// Launch the feature x token tile GEMM W [F, d] . T [B, d]^T with epilogue e.
// aux: the [B, F]-sized bf16 tensor the epilogue reads (AUX_LOAD) or writes
// (AUX_STORE) through the 64 KiB side tile: token-major [B, F], or
// feature-major [F, pre_pitch(B)] when Epi::kAuxFeatureMajor.
template <class Epi>
int aux_tmap(CUtensorMap* m, const bf16* aux, int64_t F, int64_t B, uint32_t box_tokens) {
  if (Epi::kAuxFeatureMajor)
    return make_tmap(m, aux, F, B, TILE_M, AUX_FM_BOX_TOKENS, CU_TENSOR_MAP_SWIZZLE_128B,
                     pre_pitch(B));
  return make_tmap(m, aux, B, F, box_tokens, TILE_M, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Epilogues that bounds-check their rows (kRowGuard) take any row count on
// the paired kernel: rows past F are TMA zero fill and never stored.
template <class E, class = void>
struct RowGuard : std::false_type {};
template <class E>
struct RowGuard<E, std::void_t<decltype(E::kRowGuard)>> : std::bool_constant<E::kRowGuard> {};

// w_pitch / t_pitch: row pitch of the operands in elements (0: d, dense rows).
// The contraction runs over ceil(d / TILE_K) slabs; TMA zero-fills past d.
template <class Epi>
int launch_tile_gemm(const bf16* w, const bf16* tok, int64_t F, int64_t B, int64_t d,
                     const Epi& e, bool use_tc, cudaStream_t stream, int timer = -1,
                     const bf16* aux = nullptr, int64_t w_pitch = 0, int64_t t_pitch = 0) {
  const int m_tiles = static_cast<int>((F + TILE_M - 1) / TILE_M);
  const int n_tiles = static_cast<int>((B + TILE_N - 1) / TILE_N);
  const int k_blocks = static_cast<int>((d + TILE_K - 1) / TILE_K);
  if (use_tc) {
    constexpr size_t smem = TcConfig<Epi::kAux>::SMEM;
    CUtensorMap tm_w, tm_t, tm_aux;
    SAE_TRY(make_tmap(&tm_w, w, F, d, TILE_M, TILE_K, CU_TENSOR_MAP_SWIZZLE_128B,
                      static_cast<uint64_t>(w_pitch)));
    SAE_TRY(make_tmap(&tm_t, tok, B, d, TILE_N, TILE_K, CU_TENSOR_MAP_SWIZZLE_128B,
                      static_cast<uint64_t>(t_pitch)));
    if (Epi::kAux != AUX_NONE) {
      if (aux == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "tile GEMM side tensor is NULL");
      SAE_TRY(aux_tmap<Epi>(&tm_aux, aux, F, B, TILE_N));
    } else {
      tm_aux = tm_w;
    }
    // Kernel attributes and the cluster occupancy belong to the current
    // device's context: set up once per device.
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return fail(SAE_ERR_CUDA, "no usable current device");
    if ((F % (2 * TILE_M) == 0 || RowGuard<Epi>::value) && pair_mode_enabled()) {
      // Paired CTAs: one 256-feature x 256-token tile per cluster of two.
      constexpr size_t smem2 = Tc2Config<Epi::kAux>::SMEM;
      static std::once_flag attr2_once[kMaxDevices];
      static int max_clusters_of[kMaxDevices] = {};
      std::call_once(attr2_once[dev], [dev] {
        cudaFuncSetAttribute(tc2_tile_gemm<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem2));
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(2 * std::max(1, device_info().sm_count / 2));
        lc.blockDim = dim3(TC2_THREADS);
        lc.dynamicSmemBytes = smem2;
        cudaLaunchAttribute at;
        at.id = cudaLaunchAttributeClusterDimension;
        at.val.clusterDim.x = 2;
        at.val.clusterDim.y = 1;
        at.val.clusterDim.z = 1;
        lc.attrs = &at;
        lc.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, tc2_tile_gemm<Epi>, &lc) != cudaSuccess) n = 0;
        cudaGetLastError();
        max_clusters_of[dev] = n;
      });
      const int max_clusters = max_clusters_of[dev];
      if (max_clusters > 0) {
        // Each CTA of the pair loads half of the 256-token slab.
        CUtensorMap tm_t_half, tm_aux2 = tm_aux;
        SAE_TRY(make_tmap(&tm_t_half, tok, B, d, TILE_N / 2, TILE_K, CU_TENSOR_MAP_SWIZZLE_128B,
                          static_cast<uint64_t>(t_pitch)));
        // Side-tile stores go out in 128-token slabs.
        if (Epi::kAux == AUX_STORE)
          SAE_TRY(aux_tmap<Epi>(&tm_aux2, aux, F, B, TC2_STORE_ROWS));
        const int m_pairs = static_cast<int>((F + 2 * TILE_M - 1) / (2 * TILE_M));
        const int total_pairs = m_pairs * n_tiles;
        const int clusters = std::min(total_pairs, max_clusters);
        if (timer >= 0) timer_begin(timer, stream);
        tc2_tile_gemm<Epi><<<2 * clusters, TC2_THREADS, smem2, stream>>>(
            tm_w, tm_t_half, tm_aux2, m_pairs, n_tiles, k_blocks, raster_group(), e);
        const int rc = check_launch("tc2_tile_gemm");
        if (timer >= 0) timer_end(timer, stream);
        return rc;
      }
    }
    static std::once_flag attr_once[kMaxDevices];
    std::call_once(attr_once[dev], [] {
      cudaFuncSetAttribute(tc_tile_gemm<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
    });
    const int total = m_tiles * n_tiles;
    const int grid = std::min(total, device_info().sm_count);
    if (timer >= 0) timer_begin(timer, stream);
    tc_tile_gemm<Epi><<<grid, TC_THREADS, smem, stream>>>(tm_w, tm_t, tm_aux, m_tiles, n_tiles,
                                                          k_blocks, raster_group(), e);
    const int rc = check_launch("tc_tile_gemm");
    if (timer >= 0) timer_end(timer, stream);
    return rc;
  }
  dim3 grid(n_tiles, m_tiles);
  if (timer >= 0) timer_begin(timer, stream);
  simt_tile_gemm<Epi><<<grid, TILE_M, 0, stream>>>(w, tok, static_cast<int>(F),
                                                   static_cast<int>(B), static_cast<int>(d), e);
  const int rc = check_launch("simt_tile_gemm");
  if (timer >= 0) timer_end(timer, stream);
  return rc;
}

// C = alpha * A B^T + beta * C (+ bias) on the tcgen05 tile GEMM. A [M, K] and
// B [N, K] bf16, K-major, rows lda / ldb elements apart (multiples of 8, bases
// 16-byte aligned); C row-major with rows ldc apart, fp32 or bf16.
int tc_store_gemm(int64_t M, int64_t N, int64_t K, const bf16* A, int64_t lda, const bf16* B,
                  int64_t ldb, void* C, int64_t ldc, int c_bf16, float alpha, float beta,
                  const float* bias, int bias_per_row, cudaStream_t stream, int timer = -1) {
  StoreEpi e{};
  e.c = C;
  e.ldc = ldc;
  e.rows = M;
  e.cols = N;
  e.alpha = alpha;
  e.beta = beta;
  e.bias = bias;
  e.bias_per_row = bias_per_row;
  e.c_bf16 = c_bf16;
  const int64_t eb = c_bf16 ? 2 : 4;
  e.vec = (aligned16(C) && (ldc * eb) % 16 == 0) ? 1 : 0;
  return launch_tile_gemm(A, B, M, N, K, e, true, stream, timer, nullptr, lda, ldb);
}

int transpose_bf16(const bf16* src, int64_t rows, int64_t cols, int64_t lds, bf16* dst,
                   int64_t ldd, cudaStream_t stream);

// SAE_B200_GEMM_SIMT=1 keeps sae_b200_gemm on CUDA cores.
bool gemm_simt_forced() {
  static const bool on = [] {
    const char* v = std::getenv("SAE_B200_GEMM_SIMT");
    return v != nullptr && v[0] == '1';
  }();
  return on;
}

// Products the tile GEMM takes: bf16 operands stored K-major (contiguous
// contraction dimension, 16-byte aligned bases and row pitches), an output
// with one unit stride, and sizes worth a persistent tensor-core launch.
bool gemm_tc_eligible(int64_t M, int64_t N, int64_t K, const void* A, int a_dtype, int64_t sam,
                      int64_t sak, const void* B, int b_dtype, int64_t sbn, int64_t sbk,
                      int64_t scm, int64_t scn) {
  if (gemm_simt_forced() || device_info().major != 10) return false;
  if (a_dtype != SAE_DTYPE_BF16 || b_dtype != SAE_DTYPE_BF16) return false;
  if (M < TILE_M || N < TILE_M || K < TILE_K) return false;
  if (M > (int64_t(1) << 31) - 1 - TILE_N || N > (int64_t(1) << 31) - 1 - TILE_N) return false;
  if (sak != 1 || sbk != 1 || sam < K || sbn < K || sam % 8 != 0 || sbn % 8 != 0) return false;
  if (!aligned16(A) || !aligned16(B)) return false;
  return scn == 1 || scm == 1;
}

int grid_for(int64_t n, int threads, int per_sm = 8) {
  const int64_t want = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(std::max(1, device_info().sm_count)) * per_sm;
  return static_cast<int>(std::max<int64_t>(1, std::min(want, cap)));
}

int transpose_bf16(const bf16* src, int64_t rows, int64_t cols, int64_t lds, bf16* dst,
                   int64_t ldd, cudaStream_t stream) {
  const int vec = (aligned16(src) && aligned16(dst) && lds % 8 == 0 && ldd % 8 == 0) ? 1 : 0;
  const int64_t tiles = ((rows + TP_TILE - 1) / TP_TILE) * ((cols + TP_TILE - 1) / TP_TILE);
  const int grid = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>(tiles, int64_t(device_info().sm_count) * 8)));
  transpose_bf16_kernel<<<grid, 256, 0, stream>>>(src, rows, cols, lds, dst, ldd, vec);
  return check_launch("transpose_bf16_kernel");
}

// Scratch of the dense weight-gradient path: the dense [F, ldp] bf16 operand
// (dpre, then the gated pre), and, on the tensor-core path, xc^T and go^T
// ([d, ldp] bf16 each: the tokens become the contraction's K-major dimension).
size_t dense_scratch_need(int64_t B, int64_t d, int64_t F, bool tc) {
  const size_t ldp = static_cast<size_t>(pre_pitch(B));
  return (static_cast<size_t>(F) * ldp + (tc ? 2 * static_cast<size_t>(d) * ldp : 0)) * 2;
}

int vec_threads(int64_t d) {
  const int64_t nv = d / 8;
  return static_cast<int>(std::min<int64_t>(1024, std::max<int64_t>(32, (nv + 31) / 32 * 32)));
}

int check_model(const SaeB200Model* m, bool need_shadows) {
  if (m == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "model is NULL");
  if (m->d_in <= 0 || m->n_features <= 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "d_in and n_features must be positive");
  if (!m->W_enc || !m->b_enc || !m->W_dec_fm || !m->b_dec || !m->log_threshold)
    return fail(SAE_ERR_INVALID_ARGUMENT, "model parameter pointer is NULL");
  if (need_shadows && (!m->W_enc_bf16 || !m->W_dec_bf16))
    return fail(SAE_ERR_INVALID_ARGUMENT, "bf16 weight copies are NULL");
  return SAE_OK;
}

int check_fused_shape(const SaeB200Model* m) {
  if (m->d_in % 8 != 0 || m->d_in > 8192)
    return fail(SAE_ERR_UNSUPPORTED_SHAPE,
                "fused step needs d_in %% 8 == 0 and d_in <= 8192 (got %lld)",
                static_cast<long long>(m->d_in));
  if (m->n_features > (int64_t(1) << 30))
    return fail(SAE_ERR_UNSUPPORTED_SHAPE, "n_features too large");
  return SAE_OK;
}

int check_ws(const Layout& L, void* ws, size_t bytes) {
  if (ws == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "workspace is NULL");
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
    return fail(SAE_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  if (bytes < L.total)
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "workspace has %zu bytes, needs %zu", bytes, L.total);
  return SAE_OK;
}

int check_cfg(const SaeB200StepConfig* c) {
  if (c == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "config is NULL");
  if (c->n_tokens <= 0 || c->n_tokens > (int64_t(1) << 30))
    return fail(SAE_ERR_INVALID_ARGUMENT, "n_tokens out of range");
  if (c->accum_steps <= 0) return fail(SAE_ERR_INVALID_ARGUMENT, "accum_steps must be >= 1");
  if (c->csr_capacity < 0 || c->csr_capacity > (int64_t(1) << 31) - 1)
    return fail(SAE_ERR_INVALID_ARGUMENT, "csr_capacity out of range");
  if (!(c->ste_bandwidth > 0.f)) return fail(SAE_ERR_INVALID_ARGUMENT, "ste_bandwidth must be > 0");
  return SAE_OK;
}

}  // namespace

// =====================================================================
extern "C" {

int sae_b200_version(void) { return 1; }

int64_t sae_b200_launch_count(void) { return g_launches.load(); }

int64_t sae_b200_pre_pitch(int64_t n_tokens) { return pre_pitch(n_tokens); }

int sae_b200_set_kernel_timer(int kernel, void* start_event, void* stop_event) {
  if (kernel < 0 || kernel >= kTimers)
    return fail(SAE_ERR_INVALID_ARGUMENT, "unknown kernel id %d", kernel);
  if ((start_event == nullptr) != (stop_event == nullptr))
    return fail(SAE_ERR_INVALID_ARGUMENT, "set both timer events or neither");
  g_timer_start[kernel] = static_cast<cudaEvent_t>(start_event);
  g_timer_stop[kernel] = static_cast<cudaEvent_t>(stop_event);
  return SAE_OK;
}

const char* sae_b200_last_error(void) { return g_last_error.c_str(); }

int sae_b200_get_device_status(int* status_out, int clear) {
  if (status_out == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "status_out is NULL");
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  if (e != cudaSuccess) return fail(SAE_ERR_CUDA, "read status: %s", cudaGetErrorString(e));
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return fail(SAE_ERR_CUDA, "clear status: %s", cudaGetErrorString(e));
  }
  *status_out = v;
  return SAE_OK;
}

int sae_b200_workspace_bytes(int64_t max_tokens, int64_t d_in, int64_t n_features,
                             int64_t csr_capacity, size_t* bytes_out) {
  if (bytes_out == nullptr || max_tokens <= 0 || d_in <= 0 || n_features <= 0 || csr_capacity < 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid workspace query");
  *bytes_out = make_layout(max_tokens, d_in, n_features, csr_capacity).total;
  return SAE_OK;
}

int sae_b200_workspace_offsets(int64_t n_tokens, int64_t d_in, int64_t n_features,
                               int64_t csr_capacity, size_t* offsets_out) {
  if (offsets_out == nullptr || n_tokens <= 0 || d_in <= 0 || n_features <= 0 || csr_capacity < 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid workspace query");
  const Layout L = make_layout(n_tokens, d_in, n_features, csr_capacity);
  const size_t o[SAE_WS_N_OFFSETS] = {L.theta, L.xc,       L.pre,      L.mask,    L.go,
                                      L.tok_cnt, L.tok_sqerr, L.col_offs, L.csr_tok, L.csr_val};
  for (int i = 0; i < SAE_WS_N_OFFSETS; ++i) offsets_out[i] = o[i];
  return SAE_OK;
}

}  // extern "C"

namespace {

struct ForwardCtx {
  int64_t B, d, F;
  Layout L;
  Ws w;
  int mask_words, n_tiles;
  float go_scale;
};

int forward_checks(const SaeB200Model* model, const void* x, int x_dtype,
                   const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                   const SaeB200StepStats* stats, const float* x_hat_out, ForwardCtx* c,
                   bool need_stats = true) {
  SAE_TRY(check_model(model, true));
  SAE_TRY(check_cfg(cfg));
  SAE_TRY(check_fused_shape(model));
  if (x == nullptr || (stats == nullptr && need_stats))
    return fail(SAE_ERR_INVALID_ARGUMENT, "x/stats is NULL");
  if (x_dtype != SAE_DTYPE_F32 && x_dtype != SAE_DTYPE_BF16)
    return fail(SAE_ERR_INVALID_ARGUMENT, "x_dtype must be F32 or BF16");
  if (!aligned16(x) || !aligned16(model->W_dec_bf16) || !aligned16(model->W_enc_bf16) ||
      (x_hat_out && !aligned16(x_hat_out)))
    return fail(SAE_ERR_MISALIGNED, "x, x_hat and bf16 weights must be 16-byte aligned");
  c->B = cfg->n_tokens;
  c->d = model->d_in;
  c->F = model->n_features;
  c->L = make_layout(c->B, c->d, c->F, cfg->csr_capacity);
  SAE_TRY(check_ws(c->L, workspace, workspace_bytes));
  c->w = carve(workspace, c->L);
  c->mask_words = static_cast<int>((c->F + 31) / 32);
  c->n_tiles = static_cast<int>((c->B + TILE_N - 1) / TILE_N);
  c->go_scale = static_cast<float>(
      1.0 / (static_cast<double>(cfg->accum_steps) * static_cast<double>(c->B) *
             static_cast<double>(c->d)));
  return SAE_OK;
}

// The encoder GEMM with the JumpReLU epilogue, storing pre as PRE says.
// sbits: the sampled backward's entry bitmap (NULL: none); act_sum /
// entry_sum: per-feature totals the epilogue adds to (NULL: per-tile active
// counts into tile_cnt instead).
template <int PRE>
int launch_encoder(const SaeB200Model* model, const ForwardCtx& c, uint32_t* sbits,
                   int* act_sum, int* entry_sum, bool use_tc, cudaStream_t stream) {
  const Ws& w = c.w;
  EncodeEpiT<PRE> e{};
  e.cut = w.cut;
  e.b_enc = model->b_enc;
  e.pre = w.pre;
  e.mask = w.mask;
  e.tile_cnt = w.tile_cnt;
  e.act_sum = act_sum;
  e.entry_sum = entry_sum;
  e.sbits = sbits;
  e.n_tokens = static_cast<int>(c.B);
  e.n_features = static_cast<int>(c.F);
  e.mask_words = c.mask_words;
  e.ldp = static_cast<int>(pre_pitch(c.B));
  return launch_tile_gemm(static_cast<const bf16*>(model->W_enc_bf16), w.xc, c.F, c.B, c.d, e,
                          use_tc, stream, SAE_KERNEL_ENCODER_GEMM, w.pre);
}

// theta, xc, encoder GEMM + JumpReLU epilogue, per-feature scans -> CSR offsets.
int forward_encode(const SaeB200Model* model, const void* x, int x_dtype,
                   const SaeB200StepConfig* cfg, const ForwardCtx& c, SaeB200StepStats* stats,
                   uint8_t* fired, cudaStream_t stream) {
  const int64_t B = c.B, d = c.d, F = c.F;
  const Ws& w = c.w;
  const bool sampled = cfg->grad_feat_gemm == 0;
  // 1. theta, xc
  {
    const int g = grid_for(std::max<int64_t>(F, B * d / 8), 256);
    if (x_dtype == SAE_DTYPE_BF16)
      prep_kernel<bf16><<<g, 256, 0, stream>>>(static_cast<const bf16*>(x), model->b_dec,
                                               model->log_threshold, model->b_enc,
                                               cfg->ste_bandwidth, w.theta, w.cut, w.xc, B,
                                               static_cast<int>(d), static_cast<int>(F));
    else
      prep_kernel<float><<<g, 256, 0, stream>>>(static_cast<const float*>(x), model->b_dec,
                                                model->log_threshold, model->b_enc,
                                                cfg->ste_bandwidth, w.theta, w.cut, w.xc, B,
                                                static_cast<int>(d), static_cast<int>(F));
    SAE_TRY(check_launch("prep_kernel"));
  }
  // 2. encoder GEMM + JumpReLU epilogue
  const bool use_tc = tc_eligible(d, F, cfg->force_simt);
  if (!sampled) {
    SAE_TRY(launch_encoder<PRE_FULL>(model, c, nullptr, nullptr, nullptr, use_tc, stream));
    // per-feature scans of the per-tile counts -> CSR offsets of the active
    // entries and each tile's start inside them (the GEMM backward's CSR fill)
    scan_columns_kernel<<<grid_for(F, 256), 256, 0, stream>>>(
        w.tile_cnt, w.col_tot, fired, 2 * c.n_tiles, static_cast<int>(F));
    SAE_TRY(check_launch("scan_columns_kernel"));
    scan_offsets_kernel<<<1, 1024, 0, stream>>>(w.col_tot, w.col_offs, static_cast<int>(F),
                                                cfg->csr_capacity, stats, w.counters);
    return check_launch("scan_offsets_kernel");
  }
  // sampled backward: the epilogue adds each feature's active and entry
  // counts straight into per-feature totals (integer atomics: exact)
  if (cudaMemsetAsync(w.col_tot, 0, (2 * F + 1) * sizeof(int), stream) != cudaSuccess)
    return fail(SAE_ERR_CUDA, "count reset failed");
  if (cfg->pre_entries_only)
    SAE_TRY(launch_encoder<PRE_ENTRIES>(model, c, w.sbits, w.col_act, w.col_tot, use_tc, stream));
  else
    SAE_TRY(launch_encoder<PRE_FULL>(model, c, w.sbits, w.col_act, w.col_tot, use_tc, stream));
  // 3. CSR offsets of the entries = exclusive scan of the totals
  size_t tmp_bytes = w.order_tmp_bytes;
  if (cub::DeviceScan::ExclusiveSum(w.order_tmp, tmp_bytes, w.col_tot, w.col_offs,
                                    static_cast<int>(F + 1), stream) != cudaSuccess)
    return fail(SAE_ERR_CUDA, "CSR offset scan failed");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  count_stats_kernel<<<1, 1024, 0, stream>>>(w.col_act, w.col_offs, static_cast<int>(F),
                                             cfg->csr_capacity, stats, w.counters, fired);
  return check_launch("count_stats_kernel");
}

// Gathered decode; partial != NULL writes the shard's decoder sums and counts
// instead of the residual (dictionary-sharded step).
// Row groups per token of the decode (blocks of G x V threads):
// SAE_B200_DECODE_G=1|2|4 overrides the default.
int decode_groups(int V) {
  static const int forced = [] {
    const char* v = std::getenv("SAE_B200_DECODE_G");
    return v != nullptr ? std::atoi(v) : 0;
  }();
  if ((forced == 1 || forced == 2 || forced == 4) && forced * V <= 1024) return forced;
  return std::min(4, std::max(1, 512 / V));
}

int forward_decode(const SaeB200Model* model, const void* x, int x_dtype, const ForwardCtx& c,
                   float* x_hat_out, float* partial, cudaStream_t stream) {
  const int64_t B = c.B, d = c.d, F = c.F;
  const Ws& w = c.w;
  const int V = vec_threads(d);
  const int Gq = decode_groups(V);
  const int G = Gq >= 4 ? 4 : Gq >= 2 ? 2 : 1;   // row groups per token (instantiated: 1, 2, 4)
  // dynamic shared memory: the row groups' partial sums and, for the
  // residual, the per-column go sums and the token's x columns
  const size_t x_elem = x_dtype == SAE_DTYPE_BF16 ? 2 : 4;
  const bool residual = x != nullptr && partial == nullptr;
  const size_t dyn = static_cast<size_t>(G - 1) * V * 2 * sizeof(float4) +
                     (residual ? static_cast<size_t>(V) * (2 * sizeof(float4) + 8 * x_elem) : 0);
  // Tokens' active counts are heavy-tailed: blocks take tokens in order of
  // decreasing count, round robin (a fixed, data-determined assignment, so the
  // per-block go sums stay deterministic).
  token_count_kernel<<<grid_for(B * 32, 256), 256, 0, stream>>>(w.mask, B, c.mask_words,
                                                               w.order_k0, w.order_v0);
  SAE_TRY(check_launch("token_count_kernel"));
  size_t tmp_bytes = w.order_tmp_bytes;
  if (cub::DeviceRadixSort::SortPairsDescending(w.order_tmp, tmp_bytes, w.order_k0, w.order_k1,
                                                w.order_v0, w.order_v1, static_cast<int>(B), 0,
                                                count_key_bits(F), stream) != cudaSuccess)
    return fail(SAE_ERR_CUDA, "token order sort failed");
  g_launches.fetch_add(1, std::memory_order_relaxed);
#define SAE_DECODE(XT, GG)                                                                     \
  do {                                                                                         \
    cudaFuncSetAttribute(decode_kernel<XT, GG>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                         static_cast<int>(dyn));                                               \
    decode_kernel<XT, GG><<<DECODE_GRID, V * GG, dyn, stream>>>(                              \
        w.mask, w.pre, static_cast<const bf16*>(model->W_dec_bf16), model->b_dec,             \
        static_cast<const XT*>(x), B, static_cast<int>(d), static_cast<int>(F), c.mask_words, \
        static_cast<int>(pre_pitch(B)), c.go_scale, w.go, x_hat_out, w.tok_sqerr, w.tok_cnt,  \
        w.gosum_part, partial, w.order_v1);                                                   \
  } while (0)
  timer_begin(SAE_KERNEL_DECODE, stream);
  if (x_dtype == SAE_DTYPE_BF16) {
    if (G == 4) SAE_DECODE(bf16, 4);
    else if (G == 2) SAE_DECODE(bf16, 2);
    else SAE_DECODE(bf16, 1);
  } else {
    if (G == 4) SAE_DECODE(float, 4);
    else if (G == 2) SAE_DECODE(float, 2);
    else SAE_DECODE(float, 1);
  }
#undef SAE_DECODE
  const int rc = check_launch("decode_kernel");
  timer_end(SAE_KERNEL_DECODE, stream);
  return rc;
}

int forward_stats(const SaeB200StepConfig* cfg, const ForwardCtx& c, SaeB200StepStats* stats,
                  cudaStream_t stream) {
  forward_stats_kernel<<<1, 1024, 0, stream>>>(c.w.tok_sqerr, c.w.tok_cnt, c.B,
                                               static_cast<int>(c.d), cfg->lambda_l0, cfg->al_mu,
                                               cfg->target_l0, cfg->accum_steps, stats);
  return check_launch("forward_stats_kernel");
}

}  // namespace

extern "C" {

int sae_b200_train_forward(const SaeB200Model* model, const void* x, int x_dtype,
                           const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                           SaeB200StepStats* stats, float* x_hat_out, uint8_t* fired,
                           void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ForwardCtx c;
  SAE_TRY(forward_checks(model, x, x_dtype, cfg, workspace, workspace_bytes, stats, x_hat_out,
                         &c));
  SAE_TRY(forward_encode(model, x, x_dtype, cfg, c, stats, fired, stream));
  SAE_TRY(forward_decode(model, x, x_dtype, c, x_hat_out, nullptr, stream));
  return forward_stats(cfg, c, stats, stream);
}

int sae_b200_encode_decode(const SaeB200Model* model, const void* x, int x_dtype,
                           int64_t n_tokens, void* workspace, size_t workspace_bytes,
                           float* x_hat_out, int32_t* active_counts_out, uint8_t* fired,
                           void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (x_hat_out == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "x_hat_out is NULL");
  SaeB200StepConfig cfg{};
  cfg.n_tokens = n_tokens;
  cfg.csr_capacity = 0;
  cfg.ste_bandwidth = 1.f;
  cfg.accum_steps = 1;
  ForwardCtx c;
  SAE_TRY(forward_checks(model, x, x_dtype, &cfg, workspace, workspace_bytes, nullptr, x_hat_out,
                         &c, /*need_stats=*/false));
  // theta, xc, encoder GEMM + gate epilogue (pre, mask rows, per-tile counts)
  const int64_t B = c.B, d = c.d, F = c.F;
  const Ws& w = c.w;
  {
    const int g = grid_for(std::max<int64_t>(F, B * d / 8), 256);
    if (x_dtype == SAE_DTYPE_BF16)
      prep_kernel<bf16><<<g, 256, 0, stream>>>(static_cast<const bf16*>(x), model->b_dec,
                                               model->log_threshold, model->b_enc,
                                               0.f, w.theta, w.cut, w.xc, B,
                                               static_cast<int>(d), static_cast<int>(F));
    else
      prep_kernel<float><<<g, 256, 0, stream>>>(static_cast<const float*>(x), model->b_dec,
                                                model->log_threshold, model->b_enc,
                                                0.f, w.theta, w.cut, w.xc, B,
                                                static_cast<int>(d), static_cast<int>(F));
    SAE_TRY(check_launch("prep_kernel"));
    // pre is stored only in the 32-token words holding an active entry: the
    // decode reads it there and nowhere else
    SAE_TRY(launch_encoder<PRE_ENTRIES>(model, c, nullptr, nullptr, nullptr,
                                        tc_eligible(d, F, 0), stream));
  }
  if (fired != nullptr) {
    scan_columns_kernel<<<grid_for(F, 256), 256, 0, stream>>>(w.tile_cnt, w.col_tot, fired,
                                                              2 * c.n_tiles, static_cast<int>(F));
    SAE_TRY(check_launch("scan_columns_kernel"));
  }
  SAE_TRY(forward_decode(model, nullptr, x_dtype, c, x_hat_out, nullptr, stream));
  if (active_counts_out != nullptr) {
    const cudaError_t e = cudaMemcpyAsync(active_counts_out, w.tok_cnt, B * sizeof(int32_t),
                                          cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return fail(SAE_ERR_CUDA, "counts copy: %s", cudaGetErrorString(e));
  }
  return SAE_OK;
}

}  // extern "C"

namespace {

struct AuxLayout {
  size_t list_j, list_v, cnt, g_aux, aux_sq, keys0, keys1, vals0, vals1, count_j, offs, db_full,
      gemv_part, counter, cub_tmp, cub_bytes, total;
};

int aux_end_bit(int64_t n_dead) {
  int b = 1;
  while ((int64_t(1) << b) <= n_dead) ++b;
  return b;
}

int make_aux_layout(int64_t B, int64_t d, int64_t F, int64_t n_dead, int64_t k, AuxLayout* A) {
  *A = AuxLayout{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t items = static_cast<size_t>(B) * k;
  A->list_j = take(items * 4);
  A->list_v = take(items * 4);
  A->cnt = take(B * 4);
  A->g_aux = take(B * d * 2);
  A->aux_sq = take(B * 4);
  A->keys0 = take(items * 4);
  A->keys1 = take(items * 4);
  A->vals0 = take(items * 8);
  A->vals1 = take(items * 8);
  A->count_j = take((n_dead + 1) * 4);
  A->offs = take((n_dead + 1) * 4);
  A->db_full = take(F * 4);
  A->gemv_part = take(static_cast<size_t>(GEMV_GRID) * d * 4);
  A->counter = take(256);
  size_t sort_bytes = 0, scan_bytes = 0;
  if (cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, static_cast<uint32_t*>(nullptr),
                                      static_cast<uint32_t*>(nullptr),
                                      static_cast<uint64_t*>(nullptr),
                                      static_cast<uint64_t*>(nullptr), static_cast<int>(items),
                                      0, aux_end_bit(n_dead)) != cudaSuccess ||
      cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, static_cast<int32_t*>(nullptr),
                                    static_cast<int32_t*>(nullptr),
                                    static_cast<int>(n_dead + 1)) != cudaSuccess)
    return fail(SAE_ERR_CUDA, "temporary-storage query of the aux sort failed");
  A->cub_bytes = std::max(sort_bytes, scan_bytes);
  A->cub_tmp = take(A->cub_bytes);
  A->total = off;
  return SAE_OK;
}

int check_aux(const SaeB200Model* model, const SaeB200StepConfig* cfg, const SaeB200AuxConfig* a,
              void* aux_ws, size_t aux_bytes, AuxLayout* A) {
  if (a == nullptr || a->dead == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "aux config is NULL");
  if (a->n_dead <= 0 || a->n_dead > model->n_features || a->k < 1 || a->k > a->n_dead ||
      a->k > 4096)
    return fail(SAE_ERR_INVALID_ARGUMENT, "aux needs 1 <= k <= min(n_dead, 4096), n_dead <= F");
  if (static_cast<int64_t>(cfg->n_tokens) * a->k > (int64_t(1) << 31) - 1)
    return fail(SAE_ERR_UNSUPPORTED_SHAPE, "n_tokens * k must stay below 2^31");
  SAE_TRY(make_aux_layout(cfg->n_tokens, model->d_in, model->n_features, a->n_dead, a->k, A));
  if (aux_ws == nullptr || (reinterpret_cast<uintptr_t>(aux_ws) & 255u) != 0)
    return fail(SAE_ERR_MISALIGNED, "aux workspace must be 256-byte aligned");
  if (aux_bytes < A->total)
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "aux workspace has %zu bytes, needs %zu", aux_bytes,
                A->total);
  return SAE_OK;
}

}  // namespace

extern "C" {

int sae_b200_aux_workspace_bytes(int64_t max_tokens, int64_t d_in, int64_t n_features,
                                 int64_t max_dead, int32_t k, size_t* bytes_out) {
  if (bytes_out == nullptr || max_tokens <= 0 || d_in <= 0 || n_features <= 0 || max_dead <= 0 ||
      k < 1)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid aux workspace query");
  AuxLayout A;
  SAE_TRY(make_aux_layout(max_tokens, d_in, n_features, max_dead, k, &A));
  *bytes_out = A.total;
  return SAE_OK;
}

int sae_b200_aux_forward(const SaeB200Model* model, const void* x, int x_dtype,
                         const float* x_hat, const SaeB200StepConfig* cfg, void* workspace,
                         size_t workspace_bytes, const SaeB200AuxConfig* aux, void* aux_ws,
                         size_t aux_bytes, SaeB200StepStats* stats, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ForwardCtx c;
  SAE_TRY(forward_checks(model, x, x_dtype, cfg, workspace, workspace_bytes, stats, x_hat, &c));
  if (x_hat == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "aux needs the forward's x_hat");
  if (cfg->pre_entries_only && cfg->grad_feat_gemm == 0)
    return fail(SAE_ERR_INVALID_ARGUMENT,
                "the aux loss reads the dead features' pre: run the forward with pre_entries_only = 0");
  AuxLayout A;
  SAE_TRY(check_aux(model, cfg, aux, aux_ws, aux_bytes, &A));
  auto at = [&](size_t o) { return static_cast<uint8_t*>(aux_ws) + o; };
  int32_t* list_j = reinterpret_cast<int32_t*>(at(A.list_j));
  float* list_v = reinterpret_cast<float*>(at(A.list_v));
  int32_t* cnt = reinterpret_cast<int32_t*>(at(A.cnt));
  int32_t* count_j = reinterpret_cast<int32_t*>(at(A.count_j));
  const int n_dead = static_cast<int>(aux->n_dead);
  if (cudaMemsetAsync(count_j, 0, (n_dead + 1) * sizeof(int32_t), stream) != cudaSuccess)
    return fail(SAE_ERR_CUDA, "aux count reset failed");
  const unsigned blocks = static_cast<unsigned>((c.B + AUX_TB - 1) / AUX_TB);
  if (n_dead < 65536)   // bin counts fit 16 bits: packed histograms
    aux_select_kernel<true><<<blocks, 256, 0, stream>>>(
        c.w.pre, static_cast<int>(pre_pitch(c.B)), aux->dead, n_dead, static_cast<int>(c.F),
        aux->k, c.B, list_j, list_v, cnt, count_j);
  else
    aux_select_kernel<false><<<blocks, 256, 0, stream>>>(
        c.w.pre, static_cast<int>(pre_pitch(c.B)), aux->dead, n_dead, static_cast<int>(c.F),
        aux->k, c.B, list_j, list_v, cnt, count_j);
  SAE_TRY(check_launch("aux_select_kernel"));
  const float g_scale = static_cast<float>(
      2.0 * aux->coeff / (static_cast<double>(c.B) * c.d * cfg->accum_steps));
  const int V = vec_threads(c.d);
  bf16* g_aux = reinterpret_cast<bf16*>(at(A.g_aux));
  float* aux_sq = reinterpret_cast<float*>(at(A.aux_sq));
  if (x_dtype == SAE_DTYPE_BF16)
    aux_decode_kernel<bf16><<<DECODE_GRID, V, 0, stream>>>(
        list_j, list_v, cnt, aux->dead, static_cast<int>(c.F), aux->k,
        static_cast<const bf16*>(model->W_dec_bf16), static_cast<const bf16*>(x), x_hat, c.B,
        static_cast<int>(c.d), g_scale, g_aux, aux_sq);
  else
    aux_decode_kernel<float><<<DECODE_GRID, V, 0, stream>>>(
        list_j, list_v, cnt, aux->dead, static_cast<int>(c.F), aux->k,
        static_cast<const bf16*>(model->W_dec_bf16), static_cast<const float*>(x), x_hat, c.B,
        static_cast<int>(c.d), g_scale, g_aux, aux_sq);
  SAE_TRY(check_launch("aux_decode_kernel"));
  aux_stats_kernel<<<1, 1024, 0, stream>>>(aux_sq, c.B, static_cast<int>(c.d), aux->coeff,
                                           cfg->accum_steps, stats);
  return check_launch("aux_stats_kernel");
}

int sae_b200_aux_backward(const SaeB200Model* model, const SaeB200Grads* grads,
                          const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                          const SaeB200AuxConfig* aux, void* aux_ws, size_t aux_bytes,
                          void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  SAE_TRY(check_model(model, true));
  SAE_TRY(check_cfg(cfg));
  SAE_TRY(check_fused_shape(model));
  if (grads == nullptr || !grads->W_enc || !grads->b_enc || !grads->b_dec)
    return fail(SAE_ERR_INVALID_ARGUMENT, "gradient pointer is NULL");
  const int64_t B = cfg->n_tokens, d = model->d_in, F = model->n_features;
  const Layout L = make_layout(B, d, F, cfg->csr_capacity);
  SAE_TRY(check_ws(L, workspace, workspace_bytes));
  const Ws w = carve(workspace, L);
  AuxLayout A;
  SAE_TRY(check_aux(model, cfg, aux, aux_ws, aux_bytes, &A));
  auto at = [&](size_t o) { return static_cast<uint8_t*>(aux_ws) + o; };
  const int n_dead = static_cast<int>(aux->n_dead);
  const int items = static_cast<int>(B * aux->k);
  uint32_t* keys0 = reinterpret_cast<uint32_t*>(at(A.keys0));
  uint32_t* keys1 = reinterpret_cast<uint32_t*>(at(A.keys1));
  uint64_t* vals0 = reinterpret_cast<uint64_t*>(at(A.vals0));
  uint64_t* vals1 = reinterpret_cast<uint64_t*>(at(A.vals1));
  int32_t* count_j = reinterpret_cast<int32_t*>(at(A.count_j));
  int32_t* offs = reinterpret_cast<int32_t*>(at(A.offs));
  float* db_full = reinterpret_cast<float*>(at(A.db_full));
  int* counter = reinterpret_cast<int*>(at(A.counter));
  // 1. entries sorted by dead index (stable: tokens ascend within a feature)
  aux_pack_kernel<<<grid_for(items, 256), 256, 0, stream>>>(
      reinterpret_cast<const int32_t*>(at(A.list_j)), reinterpret_cast<const float*>(at(A.list_v)),
      reinterpret_cast<const int32_t*>(at(A.cnt)), B, aux->k, n_dead, keys0, vals0);
  SAE_TRY(check_launch("aux_pack_kernel"));
  size_t tmp = A.cub_bytes;
  if (cub::DeviceRadixSort::SortPairs(at(A.cub_tmp), tmp, keys0, keys1, vals0, vals1, items, 0,
                                      aux_end_bit(n_dead), stream) != cudaSuccess)
    return fail(SAE_ERR_CUDA, "aux sort failed");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  tmp = A.cub_bytes;
  if (cub::DeviceScan::ExclusiveSum(at(A.cub_tmp), tmp, count_j, offs, n_dead + 1, stream) !=
      cudaSuccess)
    return fail(SAE_ERR_CUDA, "aux scan failed");
  g_launches.fetch_add(1, std::memory_order_relaxed);
  // 2. per dead feature: dpre, dW_enc, dW_dec, b_enc -- the sampled backward's
  //    kernel over the aux entries (all "active", no STE band), adding to the
  //    main step's gradients; its db goes to db_full for the b_dec term
  if (cudaMemsetAsync(db_full, 0, F * sizeof(float), stream) != cudaSuccess ||
      cudaMemsetAsync(counter, 0, sizeof(int), stream) != cudaSuccess)
    return fail(SAE_ERR_CUDA, "aux reset failed");
  int* tok2 = reinterpret_cast<int*>(keys0);          // free after the sort
  uint32_t* val2 = reinterpret_cast<uint32_t*>(vals0);
  aux_unpack_kernel<<<grid_for(items, 256), 256, 0, stream>>>(vals1, offs, n_dead, tok2, val2);
  SAE_TRY(check_launch("aux_unpack_kernel"));
  launch_sampled(offs, tok2, val2, reinterpret_cast<const bf16*>(at(A.g_aux)), w.xc,
                 static_cast<const bf16*>(model->W_dec_bf16), w.theta, n_dead,
                 static_cast<int>(B), static_cast<int>(d), cfg->ste_bandwidth, 1,
                 cfg->train_decoder ? grads->W_dec_fm : nullptr, grads->W_enc,
                 grads->log_threshold, grads->b_enc, db_full, counter, nullptr, aux->dead, 0,
                 stream);
  SAE_TRY(check_launch("sampled_backward_kernel (aux)"));
  // 3. b_dec: minus the aux encoder term -(sum dpre_aux) W_enc
  float* gemv_part = reinterpret_cast<float*>(at(A.gemv_part));
  bdec_gemv_kernel<<<GEMV_GRID, vec_threads(d), 0, stream>>>(
      db_full, static_cast<const bf16*>(model->W_enc_bf16), static_cast<int>(F),
      static_cast<int>(d), gemv_part);
  SAE_TRY(check_launch("bdec_gemv_kernel"));
  bdec_grad_kernel<<<static_cast<unsigned>((d + 31) / 32), 1024, 0, stream>>>(
      w.gosum_part, 0, gemv_part, GEMV_GRID, static_cast<int>(d), 1, grads->b_dec);
  return check_launch("bdec_grad_kernel");
}

int64_t sae_b200_shard_exchange_floats(int64_t n_tokens, int64_t d_in) {
  if (n_tokens <= 0 || d_in <= 0) return 0;
  return n_tokens * d_in + n_tokens;
}

int sae_b200_peer_buffer_bytes(int64_t max_tokens, int64_t d_in, int64_t n_features,
                               int64_t csr_capacity, size_t* bytes_out,
                               uint64_t* exchange_offset_out, uint64_t* flags_offset_out) {
  if (bytes_out == nullptr || exchange_offset_out == nullptr || flags_offset_out == nullptr ||
      max_tokens <= 0 || d_in <= 0 || n_features <= 0 || csr_capacity < 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid peer buffer query");
  const size_t ws = make_layout(max_tokens, d_in, n_features, csr_capacity).total;
  const size_t ex = align_up(ws, 256);
  const size_t fl = align_up(ex + static_cast<size_t>(max_tokens) * (d_in + 1) * 4, 256);
  *exchange_offset_out = ex;
  *flags_offset_out = fl;
  *bytes_out = fl + 256;
  return SAE_OK;
}

int sae_b200_peer_alloc(size_t bytes, void** ptr_out, void* handle_out) {
  if (ptr_out == nullptr || handle_out == nullptr || bytes == 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid peer allocation");
  static_assert(sizeof(cudaIpcMemHandle_t) == SAE_PEER_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(SAE_ERR_CUDA, "peer buffer cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(SAE_ERR_CUDA, "peer buffer IPC handle: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return SAE_OK;
}

int sae_b200_peer_open(const void* handle, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid peer handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(SAE_ERR_CUDA, "peer buffer open: %s", cudaGetErrorString(e));
  return SAE_OK;
}

int sae_b200_peer_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? SAE_OK : fail(SAE_ERR_CUDA, "peer close: %s", cudaGetErrorString(e));
}

int sae_b200_peer_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? SAE_OK : fail(SAE_ERR_CUDA, "peer free: %s", cudaGetErrorString(e));
}

int sae_b200_shard_forward_p2p(const SaeB200Model* model, const void* x, int x_dtype,
                               const SaeB200StepConfig* cfg, const SaeB200Peers* peers,
                               SaeB200StepStats* stats, uint8_t* fired, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (peers == nullptr || peers->world < 1 || peers->world > SAE_MAX_PEERS || peers->rank < 0 ||
      peers->rank >= peers->world)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid peer set");
  for (int p = 0; p < peers->world; ++p)
    if (peers->base[p] == nullptr || (reinterpret_cast<uintptr_t>(peers->base[p]) & 255u) != 0)
      return fail(SAE_ERR_MISALIGNED, "peer buffer %d is NULL or not 256-byte aligned", p);
  char* own = static_cast<char*>(peers->base[peers->rank]);
  ForwardCtx c;
  SAE_TRY(forward_checks(model, x, x_dtype, cfg, own, peers->exchange_offset, stats, nullptr, &c));
  if (peers->flags_offset < peers->exchange_offset + static_cast<uint64_t>(c.B) * (c.d + 1) * 4)
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "peer exchange region too small for %lld tokens",
                static_cast<long long>(c.B));
  float* exchange = reinterpret_cast<float*>(own + peers->exchange_offset);
  SAE_TRY(forward_encode(model, x, x_dtype, cfg, c, stats, fired, stream));
  SAE_TRY(forward_decode(model, x, x_dtype, c, nullptr, exchange, stream));
  // go-sum rows no rank writes (DECODE_GRID not a multiple of world) stay zero
  const int gp = DECODE_GRID / peers->world;
  const size_t used = static_cast<size_t>(gp) * peers->world;
  if (used < static_cast<size_t>(DECODE_GRID) &&
      cudaMemsetAsync(c.w.gosum_part + used * c.d, 0, (DECODE_GRID - used) * c.d * 4, stream) !=
          cudaSuccess)
    return fail(SAE_ERR_CUDA, "go-sum reset failed");
  PeerArgs a{};
  for (int p = 0; p < peers->world; ++p) a.base[p] = static_cast<char*>(peers->base[p]);
  a.rank = peers->rank;
  a.world = peers->world;
  a.epoch = peers->epoch;
  a.exchange_off = peers->exchange_offset;
  a.flags_off = peers->flags_offset;
  a.go_off = c.L.go;
  a.tok_sqerr_off = c.L.tok_sqerr;
  a.tok_cnt_off = c.L.tok_cnt;
  a.gosum_off = c.L.gosum_part;
  timer_begin(SAE_KERNEL_EXCHANGE, stream);
  peer_barrier_kernel<<<1, 32, 0, stream>>>(a, 0);
  SAE_TRY(check_launch("peer_barrier_kernel"));
  const int64_t lo = c.B * peers->rank / peers->world;
  const int64_t hi = c.B * (peers->rank + 1) / peers->world;
  const int V = vec_threads(c.d);
  if (x_dtype == SAE_DTYPE_BF16)
    exchange_reduce_kernel<bf16><<<gp, V, 0, stream>>>(a, static_cast<const bf16*>(x),
                                                       model->b_dec, c.B, static_cast<int>(c.d),
                                                       c.go_scale, lo, hi);
  else
    exchange_reduce_kernel<float><<<gp, V, 0, stream>>>(a, static_cast<const float*>(x),
                                                        model->b_dec, c.B, static_cast<int>(c.d),
                                                        c.go_scale, lo, hi);
  SAE_TRY(check_launch("exchange_reduce_kernel"));
  peer_barrier_kernel<<<1, 32, 0, stream>>>(a, 1);
  const int rc = check_launch("peer_barrier_kernel");
  timer_end(SAE_KERNEL_EXCHANGE, stream);
  SAE_TRY(rc);
  return forward_stats(cfg, c, stats, stream);
}

int sae_b200_shard_forward(const SaeB200Model* model, const void* x, int x_dtype,
                           const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                           SaeB200StepStats* stats, uint8_t* fired, float* exchange,
                           void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ForwardCtx c;
  SAE_TRY(forward_checks(model, x, x_dtype, cfg, workspace, workspace_bytes, stats, nullptr, &c));
  if (exchange == nullptr || !aligned16(exchange))
    return fail(SAE_ERR_MISALIGNED, "exchange must be a 16-byte aligned device buffer");
  SAE_TRY(forward_encode(model, x, x_dtype, cfg, c, stats, fired, stream));
  return forward_decode(model, x, x_dtype, c, nullptr, exchange, stream);
}

int sae_b200_shard_finish_forward(const SaeB200Model* model, const void* x, int x_dtype,
                                  const SaeB200StepConfig* cfg, void* workspace,
                                  size_t workspace_bytes, SaeB200StepStats* stats,
                                  const float* exchange, float* x_hat_out, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  ForwardCtx c;
  SAE_TRY(forward_checks(model, x, x_dtype, cfg, workspace, workspace_bytes, stats, x_hat_out,
                         &c));
  if (exchange == nullptr || !aligned16(exchange))
    return fail(SAE_ERR_MISALIGNED, "exchange must be a 16-byte aligned device buffer");
  const int V = vec_threads(c.d);
  const Ws& w = c.w;
  if (x_dtype == SAE_DTYPE_BF16)
    residual_kernel<bf16><<<DECODE_GRID, V, 0, stream>>>(
        exchange, model->b_dec, static_cast<const bf16*>(x), c.B, static_cast<int>(c.d),
        c.go_scale, w.go, x_hat_out, w.tok_sqerr, w.tok_cnt, w.gosum_part);
  else
    residual_kernel<float><<<DECODE_GRID, V, 0, stream>>>(
        exchange, model->b_dec, static_cast<const float*>(x), c.B, static_cast<int>(c.d),
        c.go_scale, w.go, x_hat_out, w.tok_sqerr, w.tok_cnt, w.gosum_part);
  SAE_TRY(check_launch("residual_kernel"));
  return forward_stats(cfg, c, stats, stream);
}

// bdec_owner = 0 (dictionary shards other than the first): the b_dec gradient
// gets only this shard's encoder term, overwriting; the shards' values are then
// summed across GPUs, with the go sum and the accumulated value counted once.
static int backward_common(const SaeB200Model* model, const SaeB200Grads* grads,
                           const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                           SaeB200StepStats* stats, bf16* dense_scratch,
                           size_t dense_scratch_bytes, cudaStream_t stream, int bdec_owner = 1) {
  SAE_TRY(check_model(model, true));
  SAE_TRY(check_cfg(cfg));
  SAE_TRY(check_fused_shape(model));
  if (grads == nullptr || stats == nullptr || !grads->W_enc || !grads->b_enc || !grads->b_dec ||
      !grads->log_threshold)
    return fail(SAE_ERR_INVALID_ARGUMENT, "gradient pointer is NULL");
  if (cfg->train_decoder && grads->W_dec_fm == nullptr)
    return fail(SAE_ERR_INVALID_ARGUMENT, "W_dec gradient is NULL with train_decoder set");
  if (dense_scratch != nullptr && cfg->pre_entries_only && cfg->grad_feat_gemm == 0)
    return fail(SAE_ERR_INVALID_ARGUMENT,
                "the dense backward reads all of pre: run the forward with pre_entries_only = 0");
  const int64_t B = cfg->n_tokens, d = model->d_in, F = model->n_features;
  const Layout L = make_layout(B, d, F, cfg->csr_capacity);
  SAE_TRY(check_ws(L, workspace, workspace_bytes));
  // the dense weight gradients run on the tcgen05 tile GEMM unless the caller
  // asked for CUDA cores (or the device is not an sm_100)
  const bool dense_tc = !cfg->force_simt && device_info().major == 10;
  if (dense_scratch != nullptr && dense_scratch_bytes < dense_scratch_need(B, d, F, dense_tc))
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "dense_scratch has %zu bytes, needs %zu",
                dense_scratch_bytes, dense_scratch_need(B, d, F, dense_tc));
  const Ws w = carve(workspace, L);
  const int n_tiles = static_cast<int>((B + TILE_N - 1) / TILE_N);
  const int acc = cfg->accumulate ? 1 : 0;
  float* g_wdec = cfg->train_decoder ? grads->W_dec_fm : nullptr;
  const int thr = vec_threads(d);

  // Sampled backward (cfg->grad_feat_gemm == 0): grad_feat only on the active
  // and in-band entries; otherwise the dense tcgen05 grad_feat GEMM with the
  // STE epilogue, then the CSR weight-gradient gather. Same gradients.
  if (dense_scratch == nullptr && cfg->grad_feat_gemm == 0) {
    // 1. CSR of the active and in-band entries, feature-major, token order
    csr_fill_kernel<<<grid_for(F * 8, 256, 8), 256, 0, stream>>>(
        w.pre, w.sbits, w.theta, w.col_offs, static_cast<int>(F), B,
        static_cast<int>(pre_pitch(B)), cfg->ste_bandwidth, stats, w.csr_tok, w.csr_val);
    SAE_TRY(check_launch("csr_fill_kernel"));
    // 2. sampled grad_feat + STE + weight gradients, one feature per block
    timer_begin(SAE_KERNEL_GRAD_GEMM, stream);
    launch_sampled(w.col_offs, w.csr_tok, w.csr_val, w.go, w.xc,
                   static_cast<const bf16*>(model->W_dec_bf16), w.theta, static_cast<int>(F),
                   static_cast<int>(B), static_cast<int>(d), cfg->ste_bandwidth, acc, g_wdec,
                   grads->W_enc, grads->log_threshold, grads->b_enc, w.db_enc, w.counters, stats,
                   nullptr, 1, stream, w.row_sumsq);
    const int rc = check_launch("sampled_backward_kernel");
    timer_end(SAE_KERNEL_GRAD_GEMM, stream);
    SAE_TRY(rc);
    // 3. b_dec gradient
    bdec_gemv_kernel<<<GEMV_GRID, thr, 0, stream>>>(
        w.db_enc, static_cast<const bf16*>(model->W_enc_bf16), static_cast<int>(F),
        static_cast<int>(d), w.gemv_part);
    SAE_TRY(check_launch("bdec_gemv_kernel"));
    bdec_grad_kernel<<<static_cast<unsigned>((d + 31) / 32), 1024, 0, stream>>>(
        w.gosum_part, bdec_owner ? DECODE_GRID : 0, w.gemv_part, GEMV_GRID, static_cast<int>(d),
        bdec_owner ? acc : 0, grads->b_dec, stats);
    return check_launch("bdec_grad_kernel");
  }

  // 1. dense grad_feat GEMM with the STE epilogue (+ CSR fill)
  {
    GradEpi e{};
    e.theta = w.theta;
    e.pre = w.pre;
    e.col_offs = w.col_offs;
    e.tile_base = w.tile_cnt;
    e.stats = stats;
    e.eps = cfg->ste_bandwidth;
    e.n_tokens = static_cast<int>(B);
    e.n_features = static_cast<int>(F);
    e.csr_tok = w.csr_tok;
    e.csr_val = w.csr_val;
    e.thr_part = w.thr_part;
    e.dbenc_part = w.dbenc_part;
    e.dense_dpre = dense_scratch;
    e.ldp = static_cast<int>(pre_pitch(B));
    SAE_TRY(launch_tile_gemm(static_cast<const bf16*>(model->W_dec_bf16), w.go, F, B, d, e,
                             tc_eligible(d, F, cfg->force_simt), stream, SAE_KERNEL_GRAD_GEMM,
                             w.pre));
  }
  // 2. per-feature gradients (threshold STE, b_enc)
  feature_grads_kernel<<<grid_for(F, 256), 256, 0, stream>>>(
      w.thr_part, w.dbenc_part, w.theta, 2 * n_tiles, static_cast<int>(F), cfg->ste_bandwidth, acc,
      grads->log_threshold, grads->b_enc, w.db_enc);
  SAE_TRY(check_launch("feature_grads_kernel"));
  // 3. b_dec gradient
  bdec_gemv_kernel<<<GEMV_GRID, thr, 0, stream>>>(w.db_enc, static_cast<const bf16*>(model->W_enc_bf16),
                                                  static_cast<int>(F), static_cast<int>(d),
                                                  w.gemv_part);
  SAE_TRY(check_launch("bdec_gemv_kernel"));
  bdec_grad_kernel<<<static_cast<unsigned>((d + 31) / 32), 1024, 0, stream>>>(
      w.gosum_part, bdec_owner ? DECODE_GRID : 0, w.gemv_part, GEMV_GRID, static_cast<int>(d),
      bdec_owner ? acc : 0, grads->b_dec);
  SAE_TRY(check_launch("bdec_grad_kernel"));
  // 4. weight gradients
  if (dense_scratch == nullptr) {
    // Features have few active tokens each (tens), so one row group is best;
    // the split variants serve dictionaries with very busy features.
    const int G = cfg->n_tokens / std::max<int64_t>(1, F) > 64 ? 2 : 1;
    const size_t dyn = static_cast<size_t>(G - 1) * thr * 4 * sizeof(float4);
    const int grid = device_info().sm_count * 8;
#define SAE_SCATTER(GG)                                                                        \
  scatter_weight_grads_kernel<GG><<<grid, thr * GG, dyn, stream>>>(                           \
      w.col_offs, w.csr_tok, w.csr_val, w.go, w.xc, static_cast<int>(F), static_cast<int>(d), \
      acc, g_wdec, grads->W_enc, w.counters, stats)
    if (G >= 4) SAE_SCATTER(4);
    else if (G >= 2) SAE_SCATTER(2);
    else SAE_SCATTER(1);
#undef SAE_SCATTER
    return check_launch("scatter_weight_grads_kernel");
  }
  // dense fallback: dW_enc = dpre^T xc, dW_dec = acts^T go, contractions over
  // the tokens. dense_scratch holds [F, ldp] (feature-major, like pre), whose
  // rows are already K-major; xc and go [B, d] are transposed to [d, ldp].
  if (dense_tc) {
    const int64_t ldp = pre_pitch(B);
    bf16* xcT = dense_scratch + static_cast<size_t>(F) * ldp;
    bf16* goT = xcT + static_cast<size_t>(d) * ldp;
    SAE_TRY(transpose_bf16(w.xc, B, d, d, xcT, ldp, stream));
    SAE_TRY(tc_store_gemm(F, d, B, dense_scratch, ldp, xcT, ldp, grads->W_enc, d, 0, 1.f,
                          acc ? 1.f : 0.f, nullptr, 0, stream, SAE_KERNEL_DENSE_WGRAD));
    if (g_wdec != nullptr) {
      gated_pre_kernel<<<grid_for(B * F, 256), 256, 0, stream>>>(w.pre, w.theta, B, F, ldp,
                                                                 dense_scratch);
      SAE_TRY(check_launch("gated_pre_kernel"));
      SAE_TRY(transpose_bf16(w.go, B, d, d, goT, ldp, stream));
      SAE_TRY(tc_store_gemm(F, d, B, dense_scratch, ldp, goT, ldp, g_wdec, d, 0, 1.f,
                            acc ? 1.f : 0.f, nullptr, 0, stream));
    }
    return SAE_OK;
  }
  {
    dim3 grid(static_cast<unsigned>((d + GG_T - 1) / GG_T), static_cast<unsigned>((F + GG_T - 1) / GG_T));
    const int64_t ldp = pre_pitch(B);
    gemm_generic_kernel<bf16, bf16, float><<<grid, 256, 0, stream>>>(
        F, d, B, 1.f, dense_scratch, ldp, 1, w.xc, 1, d, acc ? 1.f : 0.f, grads->W_enc, d, 1,
        nullptr);
    SAE_TRY(check_launch("gemm_generic_kernel(dW_enc)"));
    if (g_wdec != nullptr) {
      gated_pre_kernel<<<grid_for(B * F, 256), 256, 0, stream>>>(w.pre, w.theta, B, F, ldp,
                                                                 dense_scratch);
      SAE_TRY(check_launch("gated_pre_kernel"));
      gemm_generic_kernel<bf16, bf16, float><<<grid, 256, 0, stream>>>(
          F, d, B, 1.f, dense_scratch, ldp, 1, w.go, 1, d, acc ? 1.f : 0.f, g_wdec, d, 1,
          nullptr);
      SAE_TRY(check_launch("gemm_generic_kernel(dW_dec)"));
    }
  }
  return SAE_OK;
}

int sae_b200_train_backward(const SaeB200Model* model, const SaeB200Grads* grads,
                            const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                            SaeB200StepStats* stats, void* stream) {
  return backward_common(model, grads, cfg, workspace, workspace_bytes, stats, nullptr, 0,
                         static_cast<cudaStream_t>(stream));
}

int sae_b200_store_full_pre(const SaeB200Model* model, const SaeB200StepConfig* cfg,
                            void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  SAE_TRY(check_model(model, true));
  SAE_TRY(check_cfg(cfg));
  SAE_TRY(check_fused_shape(model));
  ForwardCtx c;
  c.B = cfg->n_tokens;
  c.d = model->d_in;
  c.F = model->n_features;
  c.L = make_layout(c.B, c.d, c.F, cfg->csr_capacity);
  SAE_TRY(check_ws(c.L, workspace, workspace_bytes));
  c.w = carve(workspace, c.L);
  c.mask_words = static_cast<int>((c.F + 31) / 32);
  c.n_tiles = static_cast<int>((c.B + TILE_N - 1) / TILE_N);
  // the forward's xc, thresholds and gate cut values (same cfg, same
  // bandwidth) are still in the workspace; the encoder writes pre in full, the
  // mask again (same bits) and per-tile counts into scratch the sampled path
  // does not use
  return launch_encoder<PRE_FULL>(model, c, nullptr, nullptr, nullptr,
                                  tc_eligible(c.d, c.F, cfg->force_simt), stream);
}

int sae_b200_dense_scratch_bytes(int64_t n_tokens, int64_t d_in, int64_t n_features,
                                 size_t* bytes_out) {
  if (bytes_out == nullptr || n_tokens <= 0 || d_in <= 0 || n_features <= 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid dense_scratch_bytes arguments");
  *bytes_out = dense_scratch_need(n_tokens, d_in, n_features, true);
  return SAE_OK;
}

int sae_b200_train_backward_dense(const SaeB200Model* model, const SaeB200Grads* grads,
                                  const SaeB200StepConfig* cfg, void* workspace,
                                  size_t workspace_bytes, SaeB200StepStats* stats,
                                  void* dense_scratch, size_t dense_scratch_bytes, void* stream) {
  if (dense_scratch == nullptr || !aligned16(dense_scratch))
    return fail(SAE_ERR_INVALID_ARGUMENT, "dense_scratch must be a 16-byte aligned buffer");
  return backward_common(model, grads, cfg, workspace, workspace_bytes, stats,
                         static_cast<bf16*>(dense_scratch), dense_scratch_bytes,
                         static_cast<cudaStream_t>(stream));
}

int sae_b200_shard_backward(const SaeB200Model* model, const SaeB200Grads* grads,
                            const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                            SaeB200StepStats* stats, int shard_rank, void* dense_scratch,
                            size_t dense_scratch_bytes, void* stream) {
  if (shard_rank < 0) return fail(SAE_ERR_INVALID_ARGUMENT, "shard_rank must be >= 0");
  if (dense_scratch != nullptr && !aligned16(dense_scratch))
    return fail(SAE_ERR_MISALIGNED, "dense_scratch must be 16-byte aligned");
  return backward_common(model, grads, cfg, workspace, workspace_bytes, stats,
                         static_cast<bf16*>(dense_scratch), dense_scratch_bytes,
                         static_cast<cudaStream_t>(stream), shard_rank == 0 ? 1 : 0);
}

int sae_b200_grad_norm(const SaeB200Model* model, const SaeB200Grads* grads, float max_norm,
                       void* workspace, size_t workspace_bytes, SaeB200StepStats* stats,
                       void* stream_) {
  SAE_TRY(check_model(model, false));
  if (grads == nullptr || stats == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "NULL argument");
  if (workspace == nullptr || workspace_bytes < NORM_GRID * sizeof(float))
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "grad_norm needs %zu workspace bytes",
                NORM_GRID * sizeof(float));
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int64_t d = model->d_in, F = model->n_features;
  GradList gl;
  gl.p[0] = grads->W_enc;
  gl.n[0] = F * d;
  gl.p[1] = grads->b_enc;
  gl.n[1] = F;
  gl.p[2] = grads->W_dec_fm;
  gl.n[2] = F * d;
  gl.p[3] = grads->b_dec;
  gl.n[3] = d;
  gl.p[4] = grads->log_threshold;
  gl.n[4] = F;
  for (int k = 0; k < 5; ++k)
    if (gl.p[k] != nullptr && !aligned16(gl.p[k]))
      return fail(SAE_ERR_MISALIGNED, "gradient %d must be 16-byte aligned", k);
  float* part = static_cast<float*>(workspace);
  grad_sumsq_kernel<<<NORM_GRID, 512, 0, stream>>>(gl, part);
  SAE_TRY(check_launch("grad_sumsq_kernel"));
  grad_norm_final_kernel<<<1, 1024, 0, stream>>>(part, NORM_GRID, max_norm, stats);
  return check_launch("grad_norm_final_kernel");
}

int sae_b200_grad_norm_sampled(const SaeB200Model* model, const SaeB200Grads* grads,
                               const SaeB200StepConfig* cfg, const void* workspace,
                               size_t workspace_bytes, float max_norm, void* norm_workspace,
                               size_t norm_workspace_bytes, SaeB200StepStats* stats,
                               void* stream_) {
  SAE_TRY(check_model(model, false));
  SAE_TRY(check_cfg(cfg));
  if (grads == nullptr || stats == nullptr || grads->b_dec == nullptr)
    return fail(SAE_ERR_INVALID_ARGUMENT, "NULL argument");
  if (cfg->grad_feat_gemm != 0)
    return fail(SAE_ERR_INVALID_ARGUMENT,
                "grad_norm_sampled follows the sampled backward (grad_feat_gemm = 0) only");
  if (norm_workspace == nullptr || norm_workspace_bytes < NORM_GRID * sizeof(float))
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "grad_norm_sampled needs %zu workspace bytes",
                NORM_GRID * sizeof(float));
  const int64_t d = model->d_in, F = model->n_features;
  const Layout L = make_layout(cfg->n_tokens, d, F, cfg->csr_capacity);
  SAE_TRY(check_ws(L, const_cast<void*>(workspace), workspace_bytes));
  const Ws w = carve(const_cast<void*>(workspace), L);
  GradList gl{};
  gl.p[0] = grads->b_dec;
  gl.n[0] = d;
  if (!cfg->train_decoder && grads->W_dec_fm != nullptr) {   // not covered by the rows
    gl.p[1] = grads->W_dec_fm;
    gl.n[1] = F * d;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  float* part = static_cast<float*>(norm_workspace);
  grad_sumsq_rows_kernel<<<NORM_GRID, 512, 0, stream>>>(
      w.row_sumsq, F, sampled_threads(static_cast<int>(d)) / 32, gl, part);
  SAE_TRY(check_launch("grad_sumsq_rows_kernel"));
  grad_norm_final_kernel<<<1, 1024, 0, stream>>>(part, NORM_GRID, max_norm, stats);
  return check_launch("grad_norm_final_kernel");
}

int sae_b200_grad_sumsq_sampled(const SaeB200Model* model, const SaeB200Grads* grads,
                                const SaeB200StepConfig* cfg, const void* workspace,
                                size_t workspace_bytes, void* norm_workspace,
                                size_t norm_workspace_bytes, float* sumsq_out, void* stream_) {
  SAE_TRY(check_model(model, false));
  SAE_TRY(check_cfg(cfg));
  if (grads == nullptr || sumsq_out == nullptr)
    return fail(SAE_ERR_INVALID_ARGUMENT, "NULL argument");
  if (cfg->grad_feat_gemm != 0)
    return fail(SAE_ERR_INVALID_ARGUMENT,
                "grad_sumsq_sampled follows the sampled backward (grad_feat_gemm = 0) only");
  if (norm_workspace == nullptr || norm_workspace_bytes < NORM_GRID * sizeof(float))
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "grad_sumsq_sampled needs %zu workspace bytes",
                NORM_GRID * sizeof(float));
  const int64_t d = model->d_in, F = model->n_features;
  const Layout L = make_layout(cfg->n_tokens, d, F, cfg->csr_capacity);
  SAE_TRY(check_ws(L, const_cast<void*>(workspace), workspace_bytes));
  const Ws w = carve(const_cast<void*>(workspace), L);
  GradList gl{};
  gl.p[0] = grads->b_dec;   // NULL on the shards that do not count the replicated b_dec
  gl.n[0] = d;
  if (!cfg->train_decoder && grads->W_dec_fm != nullptr) {   // not covered by the rows
    gl.p[1] = grads->W_dec_fm;
    gl.n[1] = F * d;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  float* part = static_cast<float*>(norm_workspace);
  grad_sumsq_rows_kernel<<<NORM_GRID, 512, 0, stream>>>(
      w.row_sumsq, F, sampled_threads(static_cast<int>(d)) / 32, gl, part);
  SAE_TRY(check_launch("grad_sumsq_rows_kernel"));
  sum_parts_kernel<<<1, 1024, 0, stream>>>(part, NORM_GRID, sumsq_out);
  return check_launch("sum_parts_kernel");
}

int sae_b200_grad_sumsq(const SaeB200Model* model, const SaeB200Grads* grads, void* workspace,
                        size_t workspace_bytes, float* sumsq_out, void* stream_) {
  SAE_TRY(check_model(model, false));
  if (grads == nullptr || sumsq_out == nullptr)
    return fail(SAE_ERR_INVALID_ARGUMENT, "NULL argument");
  if (workspace == nullptr || workspace_bytes < NORM_GRID * sizeof(float))
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "grad_sumsq needs %zu workspace bytes",
                NORM_GRID * sizeof(float));
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int64_t d = model->d_in, F = model->n_features;
  GradList gl;
  const float* ps[5] = {grads->W_enc, grads->b_enc, grads->W_dec_fm, grads->b_dec,
                        grads->log_threshold};
  const int64_t ns[5] = {F * d, F, F * d, d, F};
  for (int k = 0; k < 5; ++k) {
    gl.p[k] = ps[k];
    gl.n[k] = ns[k];
    if (ps[k] != nullptr && !aligned16(ps[k]))
      return fail(SAE_ERR_MISALIGNED, "gradient %d must be 16-byte aligned", k);
  }
  float* part = static_cast<float*>(workspace);
  grad_sumsq_kernel<<<NORM_GRID, 512, 0, stream>>>(gl, part);
  SAE_TRY(check_launch("grad_sumsq_kernel"));
  sum_parts_kernel<<<1, 1024, 0, stream>>>(part, NORM_GRID, sumsq_out);
  return check_launch("sum_parts_kernel");
}

int sae_b200_clip_from_sumsq(const float* sumsq, float max_norm, SaeB200StepStats* stats,
                             void* stream_) {
  if (sumsq == nullptr || stats == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "NULL argument");
  grad_norm_final_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream_)>>>(sumsq, 1, max_norm,
                                                                           stats);
  return check_launch("grad_norm_final_kernel");
}

int sae_b200_adam_step(const SaeB200Model* model, const SaeB200Grads* grads,
                       const SaeB200AdamState* state, const SaeB200AdamTensor* hyper,
                       const SaeB200StepStats* stats, void* stream_) {
  SAE_TRY(check_model(model, false));
  if (grads == nullptr || state == nullptr || hyper == nullptr)
    return fail(SAE_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int64_t d = model->d_in, F = model->n_features;
  float* params[5] = {model->W_enc, model->b_enc, model->W_dec_fm, model->b_dec,
                      model->log_threshold};
  const float* gs[5] = {grads->W_enc, grads->b_enc, grads->W_dec_fm, grads->b_dec,
                        grads->log_threshold};
  bf16* shadows[5] = {static_cast<bf16*>(model->W_enc_bf16), nullptr,
                      static_cast<bf16*>(model->W_dec_bf16), nullptr, nullptr};
  const int64_t rows[5] = {F, F, F, d, F};
  const int64_t cols[5] = {d, 1, d, 1, 1};
  timer_begin(SAE_KERNEL_ADAM, stream);
  for (int k = 0; k < 5; ++k) {
    const SaeB200AdamTensor& h = hyper[k];
    if (h.skip) continue;
    if (gs[k] == nullptr || state->exp_avg[k] == nullptr || state->exp_avg_sq[k] == nullptr)
      return fail(SAE_ERR_INVALID_ARGUMENT, "tensor %d: gradient or Adam state is NULL", k);
    if (h.step < 1) return fail(SAE_ERR_INVALID_ARGUMENT, "Adam step must be >= 1");
    if (h.use_clip && stats == nullptr)
      return fail(SAE_ERR_INVALID_ARGUMENT, "use_clip needs the stats pointer");
    AdamScalars s;
    s.lr = h.lr;
    s.beta1 = h.beta1;
    s.beta2 = h.beta2;
    s.eps = h.eps;
    s.wd = h.weight_decay;
    s.grad_scale = h.grad_scale;
    s.use_clip = h.use_clip;
    const double bc1 = 1.0 - std::pow(static_cast<double>(h.beta1), h.step);
    const double bc2 = 1.0 - std::pow(static_cast<double>(h.beta2), h.step);
    s.step_size = static_cast<float>(h.lr / bc1);
    s.bc2_sqrt = static_cast<float>(std::sqrt(bc2));
    const int64_t n = rows[k] * cols[k];
    const bool row_kernel = cols[k] > 1 && cols[k] % 4 == 0 && cols[k] <= 4096 &&
                            aligned16(params[k]) && aligned16(gs[k]) &&
                            aligned16(state->exp_avg[k]) && aligned16(state->exp_avg_sq[k]) &&
                            (shadows[k] == nullptr || (reinterpret_cast<uintptr_t>(shadows[k]) & 7u) == 0);
    // wide-row kernel: VPT float4 per thread, threads per row a multiple of 32
    int vpt = 0, tpr = 0;
    if (row_kernel) {
      const int64_t nv = cols[k] / 4;
      for (const int cand : {2, 4, 1, 3, 6, 8}) {
        if (nv % cand == 0 && (nv / cand) % 32 == 0 && nv / cand <= 512) {
          vpt = cand;
          tpr = static_cast<int>(nv / cand);
          break;
        }
      }
    }
    if (row_kernel && vpt > 0) {
      const int rpb = std::max(1, 256 / tpr);   // small blocks: more of them resident per SM
      const int threads = rpb * tpr;
      const int64_t blocks_needed = (rows[k] + rpb - 1) / rpb;
      const int per_sm = std::max(1, 2048 / threads);
      const int g = static_cast<int>(
          std::min<int64_t>(blocks_needed, static_cast<int64_t>(device_info().sm_count) * per_sm));
      const int rn = h.renorm_rows ? 1 : 0;
#define SAE_ADAM_WIDE(V)                                                                    \
  adam_rows_wide_kernel<V><<<g, threads, 0, stream>>>(params[k], gs[k], state->exp_avg[k],   \
                                                      state->exp_avg_sq[k], shadows[k],     \
                                                      rows[k], static_cast<int>(cols[k]),   \
                                                      tpr, s, stats, rn)
      switch (vpt) {
        case 1: SAE_ADAM_WIDE(1); break;
        case 2: SAE_ADAM_WIDE(2); break;
        case 3: SAE_ADAM_WIDE(3); break;
        case 4: SAE_ADAM_WIDE(4); break;
        case 6: SAE_ADAM_WIDE(6); break;
        default: SAE_ADAM_WIDE(8); break;
      }
#undef SAE_ADAM_WIDE
      SAE_TRY(check_launch("adam_rows_wide_kernel"));
    } else if (row_kernel) {
      const int nv_lane = static_cast<int>((cols[k] / 4 + 31) / 32);
      const int g = grid_for(rows[k] * 32, 256);
      const int rn = h.renorm_rows ? 1 : 0;
#define SAE_ADAM_ROWS(MV)                                                                   \
  adam_rows_kernel<MV><<<g, 256, 0, stream>>>(params[k], gs[k], state->exp_avg[k],           \
                                              state->exp_avg_sq[k], shadows[k], rows[k],     \
                                              static_cast<int>(cols[k]), s, stats, rn)
      if (nv_lane <= 4) SAE_ADAM_ROWS(4);
      else if (nv_lane <= 8) SAE_ADAM_ROWS(8);
      else if (nv_lane <= 12) SAE_ADAM_ROWS(12);
      else if (nv_lane <= 16) SAE_ADAM_ROWS(16);
      else if (nv_lane <= 24) SAE_ADAM_ROWS(24);
      else SAE_ADAM_ROWS(32);
#undef SAE_ADAM_ROWS
      SAE_TRY(check_launch("adam_rows_kernel"));
    } else {
      adam_flat_kernel<<<grid_for(n, 256), 256, 0, stream>>>(params[k], gs[k], state->exp_avg[k],
                                                             state->exp_avg_sq[k], n, s, stats);
      SAE_TRY(check_launch("adam_flat_kernel"));
      if (cols[k] > 1 && h.renorm_rows) {
        renorm_rows_kernel<<<grid_for(rows[k] * 32, 256), 256, 0, stream>>>(params[k], rows[k],
                                                                            cols[k], shadows[k]);
        SAE_TRY(check_launch("renorm_rows_kernel"));
      } else if (shadows[k] != nullptr) {
        to_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(params[k], shadows[k], n);
        SAE_TRY(check_launch("to_bf16_kernel"));
      }
    }
  }
  timer_end(SAE_KERNEL_ADAM, stream);
  return SAE_OK;
}

int sae_b200_encode_pre(const SaeB200Model* model, const void* x, int x_dtype, int64_t n_tokens,
                        void* pre_out, int pre_dtype, void* xc_out, int force_simt,
                        void* workspace, size_t workspace_bytes, void* stream_) {
  SAE_TRY(check_model(model, pre_dtype == SAE_DTYPE_BF16));
  if (x == nullptr || pre_out == nullptr || n_tokens <= 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "x/pre_out NULL or n_tokens <= 0");
  if ((x_dtype != SAE_DTYPE_F32 && x_dtype != SAE_DTYPE_BF16) ||
      (pre_dtype != SAE_DTYPE_F32 && pre_dtype != SAE_DTYPE_BF16))
    return fail(SAE_ERR_INVALID_ARGUMENT, "dtype must be F32 or BF16");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int64_t B = n_tokens, d = model->d_in, F = model->n_features;
  if (pre_dtype == SAE_DTYPE_F32) {
    if (xc_out == nullptr) return fail(SAE_ERR_INVALID_ARGUMENT, "fp32 encode_pre needs xc_out");
    if (x_dtype == SAE_DTYPE_BF16)
      sub_bias_kernel<bf16, float><<<grid_for(B * d, 256), 256, 0, stream>>>(
          static_cast<const bf16*>(x), model->b_dec, static_cast<float*>(xc_out), B, d);
    else
      sub_bias_kernel<float, float><<<grid_for(B * d, 256), 256, 0, stream>>>(
          static_cast<const float*>(x), model->b_dec, static_cast<float*>(xc_out), B, d);
    SAE_TRY(check_launch("sub_bias_kernel"));
    dim3 grid(static_cast<unsigned>((F + GG_T - 1) / GG_T), static_cast<unsigned>((B + GG_T - 1) / GG_T));
    gemm_generic_kernel<float, float, float><<<grid, 256, 0, stream>>>(
        B, F, d, 1.f, static_cast<const float*>(xc_out), d, 1, model->W_enc, d, 1, 0.f,
        static_cast<float*>(pre_out), F, 1, model->b_enc);
    return check_launch("gemm_generic_kernel(encode_pre)");
  }
  // bf16: xc (bf16) then the tile GEMM with a bias-only epilogue.
  bf16* xc = static_cast<bf16*>(xc_out);
  if (xc == nullptr) {
    const Layout L = make_layout(B, d, F, 0);
    if (workspace == nullptr || workspace_bytes < L.xc + static_cast<size_t>(B * d * 2))
      return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "encode_pre needs xc_out or a workspace");
    xc = carve(workspace, L).xc;
  }
  if (x_dtype == SAE_DTYPE_BF16)
    sub_bias_kernel<bf16, bf16><<<grid_for(B * d, 256), 256, 0, stream>>>(
        static_cast<const bf16*>(x), model->b_dec, xc, B, d);
  else
    sub_bias_kernel<float, bf16><<<grid_for(B * d, 256), 256, 0, stream>>>(
        static_cast<const float*>(x), model->b_dec, xc, B, d);
  SAE_TRY(check_launch("sub_bias_kernel"));
  PreOnlyEpi e{};
  e.b_enc = model->b_enc;
  e.pre = static_cast<bf16*>(pre_out);
  e.n_tokens = static_cast<int>(B);
  e.n_features = static_cast<int>(F);
  const bool tc = tc_eligible(d, F, force_simt) && aligned16(xc) && aligned16(pre_out);
  return launch_tile_gemm(static_cast<const bf16*>(model->W_enc_bf16), xc, F, B, d, e, tc, stream,
                          -1, static_cast<const bf16*>(pre_out));
}

int sae_b200_jumprelu_forward(const void* pre, int pre_dtype, const float* log_threshold,
                              int64_t n_tokens, int64_t n_features, float* feat_out,
                              float* gate_out, void* stream_) {
  if (pre == nullptr || log_threshold == nullptr || n_tokens <= 0 || n_features <= 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid jumprelu_forward arguments");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int g = grid_for(n_tokens * n_features, 256);
  if (pre_dtype == SAE_DTYPE_BF16)
    jumprelu_fwd_kernel<bf16><<<g, 256, 0, stream>>>(static_cast<const bf16*>(pre), log_threshold,
                                                     n_tokens, n_features, feat_out, gate_out);
  else if (pre_dtype == SAE_DTYPE_F32)
    jumprelu_fwd_kernel<float><<<g, 256, 0, stream>>>(static_cast<const float*>(pre),
                                                      log_threshold, n_tokens, n_features,
                                                      feat_out, gate_out);
  else
    return fail(SAE_ERR_INVALID_ARGUMENT, "pre_dtype must be F32 or BF16");
  return check_launch("jumprelu_fwd_kernel");
}

int sae_b200_jumprelu_backward(const void* pre, int pre_dtype, const float* log_threshold,
                               int64_t n_tokens, int64_t n_features, const float* grad_feat,
                               const float* grad_gate, float eps, void* grad_pre_out,
                               float* grad_log_threshold, void* workspace, size_t workspace_bytes,
                               void* stream_) {
  if (pre == nullptr || log_threshold == nullptr || grad_log_threshold == nullptr ||
      n_tokens <= 0 || n_features <= 0 || !(eps > 0.f))
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid jumprelu_backward arguments");
  const int64_t slabs = (n_tokens + JB_TOK - 1) / JB_TOK;
  if (slabs > kMaxGridY)
    return fail(SAE_ERR_UNSUPPORTED_SHAPE,
                "jumprelu_backward takes at most %d token slabs of %d (n_tokens <= %lld)",
                kMaxGridY, JB_TOK, static_cast<long long>(kMaxGridY) * JB_TOK);
  const size_t need = static_cast<size_t>(slabs * n_features) * sizeof(float);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(SAE_ERR_WORKSPACE_TOO_SMALL, "jumprelu_backward needs %zu workspace bytes", need);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  float* part = static_cast<float*>(workspace);
  dim3 grid(static_cast<unsigned>((n_features + 31) / 32), static_cast<unsigned>(slabs));
  if (pre_dtype == SAE_DTYPE_BF16)
    jumprelu_bwd_kernel<bf16><<<grid, 256, 0, stream>>>(
        static_cast<const bf16*>(pre), log_threshold, n_tokens, n_features, grad_feat, grad_gate,
        eps, static_cast<bf16*>(grad_pre_out), part);
  else if (pre_dtype == SAE_DTYPE_F32)
    jumprelu_bwd_kernel<float><<<grid, 256, 0, stream>>>(
        static_cast<const float*>(pre), log_threshold, n_tokens, n_features, grad_feat, grad_gate,
        eps, static_cast<float*>(grad_pre_out), part);
  else
    return fail(SAE_ERR_INVALID_ARGUMENT, "pre_dtype must be F32 or BF16");
  SAE_TRY(check_launch("jumprelu_bwd_kernel"));
  jumprelu_bwd_final_kernel<<<grid_for(n_features, 256), 256, 0, stream>>>(
      part, static_cast<int>(slabs), log_threshold, n_features, eps, grad_log_threshold);
  return check_launch("jumprelu_bwd_final_kernel");
}

}  // extern "C"

// ------------------------------------------------ allocation-free variant
// Scratch for sae_b200_jumprelu_backward_static: the per-slab partial sums of
// the threshold gradient live in this fixed device array instead of a
// caller-provided workspace. It is part of the library image, so every GPU
// that loads the library holds these 4 MiB until the process exits. Host code
// must not use the symbol itself as a device pointer; it passes the address
// that cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) float g_jumprelu_bwd_scratch[SAE_JUMPRELU_BWD_STATIC_FLOATS];

namespace {

// Device address of g_jumprelu_bwd_scratch, looked up once per device (with
// that device current) on the first call made there.
int static_scratch_address(float** out) {
  static std::mutex mu;
  static float* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SAE_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(SAE_ERR_NO_DEVICE, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_jumprelu_bwd_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(SAE_ERR_CUDA, "cudaGetSymbolAddress(jumprelu scratch): %s",
                  cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return SAE_OK;
}

}  // namespace

extern "C" {

int sae_b200_jumprelu_backward_static(const void* pre, int pre_dtype, const float* log_threshold,
                                      int64_t n_tokens, int64_t n_features,
                                      const float* grad_feat, const float* grad_gate, float eps,
                                      void* grad_pre_out, float* grad_log_threshold,
                                      void* stream_) {
  if (pre == nullptr || log_threshold == nullptr || grad_log_threshold == nullptr ||
      n_tokens <= 0 || n_features <= 0 || !(eps > 0.f))
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid jumprelu_backward_static arguments");
  if (pre_dtype != SAE_DTYPE_BF16 && pre_dtype != SAE_DTYPE_F32)
    return fail(SAE_ERR_INVALID_ARGUMENT, "pre_dtype must be F32 or BF16");
  const int64_t slabs = (n_tokens + JB_TOK - 1) / JB_TOK;
  if (slabs > kMaxGridY)
    return fail(SAE_ERR_UNSUPPORTED_SHAPE,
                "jumprelu_backward_static takes at most %d token slabs of %d (n_tokens <= %lld)",
                kMaxGridY, JB_TOK, static_cast<long long>(kMaxGridY) * JB_TOK);
  if (n_features > SAE_JUMPRELU_BWD_STATIC_FLOATS ||
      slabs > SAE_JUMPRELU_BWD_STATIC_FLOATS / n_features)
    return fail(SAE_ERR_UNSUPPORTED_SHAPE,
                "jumprelu_backward_static holds at most %d partial sums: ceil(n_tokens/%d) * "
                "n_features = %lld * %lld is too large; use sae_b200_jumprelu_backward with a "
                "workspace",
                SAE_JUMPRELU_BWD_STATIC_FLOATS, JB_TOK, static_cast<long long>(slabs),
                static_cast<long long>(n_features));
  float* part = nullptr;
  SAE_TRY(static_scratch_address(&part));
  // Every (slab, feature) partial is written by the first kernel before the
  // second reads it, so nothing left over from an earlier call is ever read
  // and the array needs no clearing.
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  dim3 grid(static_cast<unsigned>((n_features + 31) / 32), static_cast<unsigned>(slabs));
  if (pre_dtype == SAE_DTYPE_BF16)
    jumprelu_bwd_kernel<bf16><<<grid, 256, 0, stream>>>(
        static_cast<const bf16*>(pre), log_threshold, n_tokens, n_features, grad_feat, grad_gate,
        eps, static_cast<bf16*>(grad_pre_out), part);
  else
    jumprelu_bwd_kernel<float><<<grid, 256, 0, stream>>>(
        static_cast<const float*>(pre), log_threshold, n_tokens, n_features, grad_feat, grad_gate,
        eps, static_cast<float*>(grad_pre_out), part);
  SAE_TRY(check_launch("jumprelu_bwd_kernel(static scratch)"));
  jumprelu_bwd_final_kernel<<<grid_for(n_features, 256), 256, 0, stream>>>(
      part, static_cast<int>(slabs), log_threshold, n_features, eps, grad_log_threshold);
  return check_launch("jumprelu_bwd_final_kernel(static scratch)");
}

int sae_b200_gemm(int64_t M, int64_t N, int64_t K, float alpha, const void* A, int a_dtype,
                  int64_t sam, int64_t sak, const void* B, int b_dtype, int64_t sbn, int64_t sbk,
                  float beta, void* C, int c_dtype, int64_t scm, int64_t scn, const float* bias_n,
                  void* stream_) {
  if (M <= 0 || N <= 0 || K < 0 || A == nullptr || B == nullptr || C == nullptr)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid gemm arguments");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (a_dtype < 0 || a_dtype > 1 || b_dtype < 0 || b_dtype > 1 || c_dtype < 0 || c_dtype > 1)
    return fail(SAE_ERR_INVALID_ARGUMENT, "gemm dtype must be F32 or BF16");
  // bf16 operands with the contraction dimension contiguous go to the tcgen05
  // tile GEMM: rows of the tile are the output's contiguous-row dimension
  // (C^T = B A^T when C is column-major).
  if (gemm_tc_eligible(M, N, K, A, a_dtype, sam, sak, B, b_dtype, sbn, sbk, scm, scn)) {
    if (scn == 1)
      return tc_store_gemm(M, N, K, static_cast<const bf16*>(A), sam,
                           static_cast<const bf16*>(B), sbn, C, scm, c_dtype == SAE_DTYPE_BF16,
                           alpha, beta, bias_n, 0, stream);
    return tc_store_gemm(N, M, K, static_cast<const bf16*>(B), sbn, static_cast<const bf16*>(A),
                         sam, C, scn, c_dtype == SAE_DTYPE_BF16, alpha, beta, bias_n, 1, stream);
  }
  dim3 grid(static_cast<unsigned>((N + GG_T - 1) / GG_T), static_cast<unsigned>((M + GG_T - 1) / GG_T));
  if (grid.y > 65535) return fail(SAE_ERR_UNSUPPORTED_SHAPE, "gemm: M too large");
  const int code = a_dtype * 4 + b_dtype * 2 + c_dtype;
#define SAE_GEMM_CASE(CODE, TA, TB, TC)                                                        \
  case CODE:                                                                                 \
    gemm_generic_kernel<TA, TB, TC><<<grid, 256, 0, stream>>>(                               \
        M, N, K, alpha, static_cast<const TA*>(A), sam, sak, static_cast<const TB*>(B), sbn, \
        sbk, beta, static_cast<TC*>(C), scm, scn, bias_n);                                   \
    break;
  switch (code) {
    SAE_GEMM_CASE(0, float, float, float)
    SAE_GEMM_CASE(1, float, float, bf16)
    SAE_GEMM_CASE(2, float, bf16, float)
    SAE_GEMM_CASE(3, float, bf16, bf16)
    SAE_GEMM_CASE(4, bf16, float, float)
    SAE_GEMM_CASE(5, bf16, float, bf16)
    SAE_GEMM_CASE(6, bf16, bf16, float)
    SAE_GEMM_CASE(7, bf16, bf16, bf16)
  }
#undef SAE_GEMM_CASE
  return check_launch("gemm_generic_kernel");
}

int sae_b200_transpose(const void* src, int dtype, int64_t rows, int64_t cols, int64_t lds,
                       void* dst, int64_t ldd, void* stream_) {
  if (src == nullptr || dst == nullptr || rows <= 0 || cols <= 0 || lds < cols || ldd < rows)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid transpose arguments");
  if (dtype != SAE_DTYPE_BF16) return fail(SAE_ERR_INVALID_ARGUMENT, "transpose takes bf16");
  return transpose_bf16(static_cast<const bf16*>(src), rows, cols, lds, static_cast<bf16*>(dst),
                        ldd, static_cast<cudaStream_t>(stream_));
}

int sae_b200_column_sum(const void* X, int x_dtype, int64_t rows, int64_t cols, float alpha,
                        float beta, float* out, void* stream_) {
  if (X == nullptr || out == nullptr || rows < 0 || cols <= 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid column_sum arguments");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int g = grid_for(cols, 256);
  if (x_dtype == SAE_DTYPE_BF16)
    column_sum_kernel<bf16><<<g, 256, 0, stream>>>(static_cast<const bf16*>(X), rows, cols, alpha,
                                                   beta, out);
  else if (x_dtype == SAE_DTYPE_F32)
    column_sum_kernel<float><<<g, 256, 0, stream>>>(static_cast<const float*>(X), rows, cols,
                                                    alpha, beta, out);
  else
    return fail(SAE_ERR_INVALID_ARGUMENT, "x_dtype must be F32 or BF16");
  return check_launch("column_sum_kernel");
}

int sae_b200_renorm_rows(float* W, int64_t rows, int64_t cols, void* shadow_bf16, void* stream_) {
  if (W == nullptr || rows <= 0 || cols <= 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid renorm_rows arguments");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  renorm_rows_kernel<<<grid_for(rows * 32, 256), 256, 0, stream>>>(W, rows, cols,
                                                                    static_cast<bf16*>(shadow_bf16));
  return check_launch("renorm_rows_kernel");
}

int sae_b200_refresh_shadow(const float* src, void* dst_bf16, int64_t n, void* stream_) {
  if (src == nullptr || dst_bf16 == nullptr || n < 0)
    return fail(SAE_ERR_INVALID_ARGUMENT, "invalid refresh_shadow arguments");
  if (n == 0) return SAE_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  to_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(src, static_cast<bf16*>(dst_bf16), n);
  return check_launch("to_bf16_kernel");
}

}  // extern "C"
