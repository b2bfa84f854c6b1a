// Feature-by-token tile GEMM with a pluggable epilogue.
//
//   D[f, t] = sum_k W[f, k] * T[t, k]        W: [F, d] bf16, T: [B, d] bf16
//
// Rows of D are dictionary features, columns are tokens. Both operands are
// K-major (d contiguous), which is the natural layout of W_enc [F, d], of the
// feature-major decoder [F, d] and of the token batches [B, d]. With features
// on the TMEM lanes, every per-feature reduction an epilogue needs (threshold
// STE sums, encoder-bias gradient, per-tile active counts) stays inside one
// thread, and per-token quantities fall out of warp ballots.
//
// Two mainloops produce the same 128 x 256 tiles and call the same epilogue:
//   * tc_tile_gemm: persistent, warp-specialised tcgen05 kernel. TMA (no
//     multicast) streams 128x64 / 256x64 bf16 slabs through a 3-4 stage
//     mbarrier ring; one thread issues tcgen05.mma into a double-buffered
//     TMEM accumulator (2 x 256 columns); four epilogue warps drain the
//     other accumulator with tcgen05.ld while the next tile accumulates. A
//     64 KiB token-major side tile can be TMA-loaded for the epilogue or
//     TMA-stored from it.
//   * simt_tile_gemm: plain CUDA-core kernel with full predication, for
//     shapes TMA cannot describe (d not a multiple of 64, F not a multiple
//     of 128) and for small problems.
#pragma once
#include <cuda.h>
#include "ptx.cuh"

namespace sae {
using bf16 = __nv_bfloat16;
}

namespace sae {

constexpr int TILE_M = 128;   // features per tile (TMEM lanes)
constexpr int TILE_N = 256;   // tokens per tile (TMEM columns per accumulator)
constexpr int TILE_K = 64;    // d per pipeline stage (one 128-byte swizzle row)
constexpr int HALF_N = TILE_N / 2;   // tokens per epilogue half: unit of the per-feature counts
constexpr int TC_A_BYTES = TILE_M * TILE_K * 2;   // 16 KiB
constexpr int TC_B_BYTES = TILE_N * TILE_K * 2;   // 32 KiB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;
constexpr int TC_THREADS = 192;   // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
constexpr int TC_GROUP_M = 16;    // default feature tiles (pairs) per rasterisation group
constexpr int TC_BARRIER_BYTES = 256;
constexpr uint32_t TC_TMEM_COLS = 2 * TILE_N;     // two fp32 accumulators

// Auxiliary 128-feature x 256-token bf16 tile (64 KiB) that rides along with
// each output tile: loaded by TMA for epilogues that read a [B, F]-sized
// tensor (AUX_LOAD), or written by the epilogue and stored by TMA for
// epilogues that produce one (AUX_STORE). Two layouts:
//  * token-major (Epi::kAuxFeatureMajor == false): one [256 tokens][128
//    features] box, no swizzle, for a token-major [B, F] global tensor;
//  * feature-major: four [128 features][64 tokens] boxes with 128-byte
//    swizzle, for a feature-major [F, ldp] global tensor. A thread that owns
//    one feature moves 8 tokens with one 16-byte shared-memory access, and
//    the swizzle spreads the 8 threads of each access phase over all banks.
enum AuxMode { AUX_NONE = 0, AUX_LOAD = 1, AUX_STORE = 2 };
constexpr int TC_AUX_BYTES = TILE_N * TILE_M * 2;
constexpr int AUX_FM_BOX_TOKENS = 64;
constexpr int AUX_FM_BOX_BYTES = TILE_M * AUX_FM_BOX_TOKENS * 2;   // 16 KiB

// Byte offset of the 16-byte group holding tokens [8 g, 8 g + 8) of feature
// row `row` in a feature-major side tile (g = 0..31).
__device__ __forceinline__ uint32_t aux_fm_offset(int row, int g) {
  return static_cast<uint32_t>((g >> 3) * AUX_FM_BOX_BYTES + row * 128 +
                               (((g & 7) ^ (row & 7)) << 4));
}

template <int AUX>
struct TcConfig {
  static constexpr int STAGES = AUX == AUX_NONE ? 4 : 3;
  static constexpr size_t SMEM = STAGES * TC_STAGE_BYTES + (AUX == AUX_NONE ? 0 : TC_AUX_BYTES) +
                                 TC_BARRIER_BYTES + 1024;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_store_2d_nocommit(const void* tmap, const void* smem_src,
                                                      int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Side-tile TMA load of the tile at (first feature f0, first token t0).
template <class Epi>
__device__ __forceinline__ void aux_load_tile(bf16* s_aux, const CUtensorMap* tm, uint64_t* bar,
                                              int f0, int t0) {
  if constexpr (Epi::kAuxFeatureMajor) {
#pragma unroll
    for (int b = 0; b < TILE_N / AUX_FM_BOX_TOKENS; ++b)
      tma_load_2d(reinterpret_cast<uint8_t*>(s_aux) + b * AUX_FM_BOX_BYTES, tm, bar,
                  t0 + b * AUX_FM_BOX_TOKENS, f0);
  } else {
    tma_load_2d(s_aux, tm, bar, f0, t0);
  }
}

// Side-tile TMA store of tokens [r0, r0 + n) of the tile (one bulk group).
// Token-major tiles use a tensor map whose box is n tokens high.
template <class Epi>
__device__ __forceinline__ void aux_store_rows(const bf16* s_aux, const CUtensorMap* tm, int f0,
                                               int t0, int r0, int n) {
  if constexpr (Epi::kAuxFeatureMajor) {
    for (int b = r0 / AUX_FM_BOX_TOKENS; b < (r0 + n) / AUX_FM_BOX_TOKENS; ++b)
      tma_store_2d_nocommit(tm, reinterpret_cast<const uint8_t*>(s_aux) + b * AUX_FM_BOX_BYTES,
                            t0 + b * AUX_FM_BOX_TOKENS, f0);
  } else {
    tma_store_2d_nocommit(tm, s_aux + r0 * TILE_M, f0, t0 + r0);
  }
  bulk_commit();
}
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

struct TileCoord {
  int m, n;
};

// Tiles are visited in groups of group_m feature tiles; inside a group the
// feature tile varies fastest, so the CTAs running at any moment share a few
// token slabs and a few weight slabs in L2. The token operand is streamed
// once per group, the weight operand about once in all.
__device__ __forceinline__ TileCoord tile_coord(int t, int m_tiles, int n_tiles, int group_m) {
  const int per_group = group_m * n_tiles;
  const int g = t / per_group;
  const int r = t - g * per_group;
  const int m0 = g * group_m;
  const int gm = min(group_m, m_tiles - m0);
  TileCoord c;
  c.m = m0 + r % gm;
  c.n = r / gm;
  return c;
}

// Epilogue contract (Epi):
//   static constexpr int kAux                   AUX_NONE / AUX_LOAD / AUX_STORE
//   begin_tile(m_tile, n_tile, row, quarter, lane, aux)   row = feature in tile;
//       aux = the tile's [TILE_N][TILE_M] bf16 shared-memory buffer, or nullptr
//       (CUDA-core path: the epilogue then uses global memory directly)
//   begin_half(h) / end_half(h)   around the chunks of tokens [128 h, 128 h + 128);
//       the paired kernel runs the two halves on different warps
//   chunk(col, v[32])   v[j] = D[row, col + j], col in {0, 32, ..., 224};
//                       called by all 32 lanes of a warp together (ballots)
//   end_tile()
template <class Epi>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_tile_gemm(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_t,
                 const __grid_constant__ CUtensorMap tm_aux, int m_tiles, int n_tiles,
                 int k_blocks, int group_m, const Epi epi) {
  constexpr int AUX = Epi::kAux;
  constexpr int STAGES = TcConfig<AUX>::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * TC_A_BYTES;
  bf16* s_aux = reinterpret_cast<bf16*>(smem + STAGES * TC_STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * TC_STAGE_BYTES +
                                               (AUX == AUX_NONE ? 0 : TC_AUX_BYTES));
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint64_t* aux_full = bars + 2 * STAGES + 5;
  uint64_t* aux_empty = bars + 2 * STAGES + 6;
  uint64_t* epi_bar = bars + 2 * STAGES + 7;   // barrier among the 128 epilogue threads
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);   // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    mbar_init(aux_full, 1);
    mbar_init(aux_empty, 4);
    mbar_init(epi_bar, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TC_TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_t);
    if (AUX != AUX_NONE) prefetch_tmap(&tm_aux);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int total = m_tiles * n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      uint32_t issued = 0, issued_parity = 0;
      bool ok = true, aux_issued = false;
      uint32_t aux_parity = 0;
      int kit = 0, it = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        const TileCoord tc = tile_coord(t, m_tiles, n_tiles, group_m);
        for (int kb = 0; kb < k_blocks; ++kb, ++kit) {
          const int s = kit % STAGES;
          const uint32_t ph = (kit / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], TC_STAGE_BYTES);
          tma_load_2d(s_a + s * TC_A_BYTES, &tm_w, &full[s], kb * TILE_K, tc.m * TILE_M);
          tma_load_2d(s_b + s * TC_B_BYTES, &tm_t, &full[s], kb * TILE_K, tc.n * TILE_N);
          issued |= 1u << s;
          issued_parity = (issued_parity & ~(1u << s)) | (ph << s);
        }
        if (AUX == AUX_LOAD && ok) {
          // After the tile's operand loads, so the previous tile's epilogue
          // (which frees the buffer) is not waited on ahead of the mainloop.
          const uint32_t ph = it & 1;
          if (!mbar_wait(aux_empty, ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(aux_full, TC_AUX_BYTES);
          aux_load_tile<Epi>(s_aux, &tm_aux, aux_full, tc.m * TILE_M, tc.n * TILE_N);
          aux_issued = true;
          aux_parity = ph;
        }
      }
      if (!ok) {
        // Unwinding: let every copy this thread started land before the CTA
        // (and its shared memory) goes away.
        for (int s = 0; s < STAGES; ++s)
          if ((issued >> s) & 1u) mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr);
        if (aux_issued) mbar_wait(aux_full, aux_parity, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------------- MMA issue
      constexpr uint32_t idesc = idesc_bf16_f32(TILE_M, TILE_N);
      bool ok = true, any_mma = false;
      int kit = 0, it = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], aph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TILE_N);
        for (int kb = 0; kb < k_blocks; ++kb, ++kit) {
          const int s = kit % STAGES;
          const uint32_t ph = (kit / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = smem_desc_k_sw128(s_a + s * TC_A_BYTES);
          const uint64_t bdesc = smem_desc_k_sw128(s_b + s * TC_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < TILE_K / 16; ++kk) {
            // 16 bf16 = 32 bytes further along the swizzled row: +2 in the
            // descriptor's 16-byte address units.
            tc_mma_bf16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          }
          any_mma = true;
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);
      }
      if (!ok && any_mma) {
        tc_commit(drain);
        mbar_wait(drain, 0, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;   // TMEM lane quarter this warp can address
    const int row = q * 32 + lane;
    const bool issuer = (warp == 2 && lane == 0);
    uint32_t epi_phase = 0;
    // All 128 epilogue threads meet here; a bounded mbarrier wait (not
    // bar.sync) so that an aborting CTA cannot strand the others.
    auto epi_sync = [&]() -> bool {
      mbar_arrive(epi_bar);
      const bool r = mbar_wait(epi_bar, epi_phase, abort_flag);
      epi_phase ^= 1;
      return r;
    };
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (AUX == AUX_STORE) {
        // The previous tile's TMA store must have finished reading the buffer.
        if (issuer) bulk_wait_read_all();
        if (!epi_sync()) break;
      }
      if (!mbar_wait(&acc_full[acc], aph, abort_flag)) break;
      if (AUX == AUX_LOAD && !mbar_wait(aux_full, it & 1, abort_flag)) break;
      tc_fence_after();
      const TileCoord tc = tile_coord(t, m_tiles, n_tiles, group_m);
      Epi e = epi;
      e.begin_tile(tc.m, tc.n, row, q, lane, AUX == AUX_NONE ? nullptr : s_aux);
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * TILE_N);
#pragma unroll 1
      for (int c = 0; c < TILE_N; c += 32) {
        if (c % (TILE_N / 2) == 0) e.begin_half(c / (TILE_N / 2));
        float v[32];
        tmem_ld_32cols(t_row + c, v);
        if (c == TILE_N - 32) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        e.chunk(c, v);
        if (c % (TILE_N / 2) == TILE_N / 2 - 32) e.end_half(c / (TILE_N / 2));
      }
      if (AUX == AUX_LOAD) {
        __syncwarp();
        if (lane == 0) mbar_arrive(aux_empty);
      }
      e.end_tile();
      if (AUX == AUX_STORE) {
        fence_proxy_async_smem();
        if (!epi_sync()) break;
        if (issuer) aux_store_rows<Epi>(s_aux, &tm_aux, tc.m * TILE_M, tc.n * TILE_N, 0, TILE_N);
      }
    }
    if (AUX == AUX_STORE && issuer) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TC_TMEM_COLS);
  }
}

// ------------------------------------------------------------------------
// Paired-CTA version (tcgen05 cta_group::2). A cluster of two CTAs computes a
// 256-feature x 256-token tile: CTA r holds feature rows [128 r, 128 r + 128)
// of the A slab and token rows [128 r, 128 r + 128) of the B slab in its own
// shared memory, and the leader (rank 0) issues one M=256, N=256 MMA per
// K step that reads both CTAs' halves and writes each CTA's 128 x 256
// accumulator into that CTA's TMEM. Per SM this moves 32 KiB per K slab
// instead of 48 KiB, and the ring gets 5-6 stages. Each CTA's epilogue is
// the same as in the single-CTA kernel (its own 128 features x 256 tokens).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (barriers other CTAs arrive on).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait_cluster(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_cluster(a, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_device_status(SAE_ERR_DEVICE_TIMEOUT);
      if (abort != nullptr) *abort = 1;
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap,
                                                 uint32_t leader_bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this offset in both CTAs once the pair's MMAs are done.
__device__ __forceinline__ void tc_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair_local(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// warps: 0 operand TMA, 1 MMA, 2 side-tile TMA, 3..10 epilogue (two groups of
// four, one per 128-token half of the tile)
constexpr int TC2_THREADS = 352;
constexpr int TC2_AUX_WARP = 2;
constexpr int TC2_EPI_WARP0 = 3;
constexpr int TC2_STORE_ROWS = 128;   // tokens per side-tile TMA store (two per tile)

__device__ __forceinline__ void bulk_wait_read_le1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

constexpr int TC2_A_BYTES = TILE_M * TILE_K * 2;      // 16 KiB: this CTA's 128 features
constexpr int TC2_B_BYTES = (TILE_N / 2) * TILE_K * 2;  // 16 KiB: this CTA's 128 tokens
constexpr int TC2_STAGE_BYTES = TC2_A_BYTES + TC2_B_BYTES;

template <int AUX>
struct Tc2Config {
  // as many 32 KiB stages as the 227 KiB of shared memory a CTA may use hold
  static constexpr int STAGES = AUX == AUX_NONE ? 7 : 5;
  static constexpr size_t SMEM = STAGES * TC2_STAGE_BYTES +
                                 (AUX == AUX_NONE ? 0 : TC_AUX_BYTES) + TC_BARRIER_BYTES + 1024;
  static_assert(SMEM <= 227 * 1024, "tile GEMM stages exceed the shared memory of a CTA");
  static_assert((2 * STAGES + 10) * 8 + 8 <= TC_BARRIER_BYTES, "barrier area too small");
};

// Pair tile t -> (feature pair index, token tile), same grouping as tile_coord.
template <class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TC2_THREADS, 1)
    tc2_tile_gemm(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_t,
                  const __grid_constant__ CUtensorMap tm_aux, int m_pairs, int n_tiles,
                  int k_blocks, int group_m, const Epi epi) {
  constexpr int AUX = Epi::kAux;
  constexpr int STAGES = Tc2Config<AUX>::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * TC2_A_BYTES;
  bf16* s_aux = reinterpret_cast<bf16*>(smem + STAGES * TC2_STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * TC2_STAGE_BYTES +
                                               (AUX == AUX_NONE ? 0 : TC_AUX_BYTES));
  uint64_t* full = bars;                        // leader: both CTAs' TMA bytes
  uint64_t* empty = bars + STAGES;              // each CTA: stage free (leader's commit)
  uint64_t* acc_full = bars + 2 * STAGES;       // each CTA: accumulator ready
  uint64_t* acc_empty = bars + 2 * STAGES + 2;  // leader: 16 epilogue warps done
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint64_t* aux_full = bars + 2 * STAGES + 5;
  uint64_t* aux_empty = bars + 2 * STAGES + 6;
  uint64_t* epi_bar = bars + 2 * STAGES + 7;    // [2]: one per epilogue half
  uint64_t* done_bar = bars + 2 * STAGES + 9;   // end-of-kernel handshake of the pair
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t peer = rank ^ 1u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 16);   // eight epilogue warps in each CTA of the pair
      mbar_init(&epi_bar[a], 128);
    }
    mbar_init(drain, 1);
    mbar_init(aux_full, 1);
    mbar_init(aux_empty, 8);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, TC_TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_t);
    if (AUX != AUX_NONE) prefetch_tmap(&tm_aux);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();   // both CTAs' barriers exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int pairs = gridDim.x >> 1;
  const int pair = blockIdx.x >> 1;
  const int total = m_pairs * n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      bool ok = true;
      int kit = 0;
      for (int t = pair; t < total && ok; t += pairs) {
        const TileCoord tc = tile_coord(t, m_pairs, n_tiles, group_m);
        const int f0 = (2 * tc.m + static_cast<int>(rank)) * TILE_M;
        const int t0 = tc.n * TILE_N + static_cast<int>(rank) * (TILE_N / 2);
        for (int kb = 0; kb < k_blocks; ++kb, ++kit) {
          const int s = kit % STAGES;
          const uint32_t ph = (kit / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t lbar = mapa_shared(smem_u32(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * TC2_STAGE_BYTES);
          tma_load_2d_pair(s_a + s * TC2_A_BYTES, &tm_w, lbar, kb * TILE_K, f0);
          tma_load_2d_pair(s_b + s * TC2_B_BYTES, &tm_t, lbar, kb * TILE_K, t0);
        }
      }
      // Operand copies of an aborted pipeline complete on the leader's full
      // barriers; the leader's MMA thread below drains them.
    }
  } else if (warp == TC2_AUX_WARP) {
    if (AUX == AUX_LOAD && lane == 0) {
      // ------------------------------------------------- side-tile producer
      // Its own thread, so waiting for the previous tile's epilogue to free
      // the buffer never holds up the operand loads of warp 0.
      uint32_t aux_parity = 0;
      bool aux_issued = false;
      int it = 0;
      for (int t = pair; t < total; t += pairs, ++it) {
        const TileCoord tc = tile_coord(t, m_pairs, n_tiles, group_m);
        const int f0 = (2 * tc.m + static_cast<int>(rank)) * TILE_M;
        const uint32_t ph = it & 1;
        if (!mbar_wait(aux_empty, ph ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(aux_full, TC_AUX_BYTES);
        aux_load_tile<Epi>(s_aux, &tm_aux, aux_full, f0, tc.n * TILE_N);
        aux_issued = true;
        aux_parity = ph;
      }
      if (aux_issued && *abort_flag) mbar_wait(aux_full, aux_parity, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // --------------------------------------------------------- MMA issue
      constexpr uint32_t idesc = idesc_bf16_f32(2 * TILE_M, TILE_N);
      bool ok = true, any_mma = false;
      int kit = 0, it = 0;
      for (int t = pair; t < total && ok; t += pairs, ++it) {
        const int acc = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait_cluster(&acc_empty[acc], aph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TILE_N);
        for (int kb = 0; kb < k_blocks; ++kb, ++kit) {
          const int s = kit % STAGES;
          const uint32_t ph = (kit / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = smem_desc_k_sw128(s_a + s * TC2_A_BYTES);
          const uint64_t bdesc = smem_desc_k_sw128(s_b + s * TC2_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < TILE_K / 16; ++kk)
            tc_mma_bf16_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          any_mma = true;
          tc_commit_pair_both(&empty[s]);
        }
        if (!ok) break;
        tc_commit_pair_both(&acc_full[acc]);
      }
      if (!ok && any_mma) {
        tc_commit_pair_local(drain);
        mbar_wait(drain, 0, nullptr);
      }
    }
  } else if (warp >= TC2_EPI_WARP0) {
    // ------------------------------------------------------------ epilogue
    // Eight warps: half h = 0 handles tokens [0, 128) of the tile, h = 1
    // tokens [128, 256); within a half, warp w reads TMEM lane quarter w % 4.
    const int h = (warp - TC2_EPI_WARP0) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool issuer = (warp == TC2_EPI_WARP0 + 4 * h) && lane == 0;
    const uint32_t leader_acc_empty0 = mapa_shared(smem_u32(&acc_empty[0]), 0);
    const uint32_t leader_acc_empty1 = mapa_shared(smem_u32(&acc_empty[1]), 0);
    uint32_t epi_phase = 0;
    auto epi_sync = [&]() -> bool {   // the 128 threads of this half
      mbar_arrive(&epi_bar[h]);
      const bool r = mbar_wait(&epi_bar[h], epi_phase, abort_flag);
      epi_phase ^= 1;
      return r;
    };
    const int c_begin = h * (TILE_N / 2);
    int it = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += pairs, ++it) {
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (AUX == AUX_STORE) {
        // this half's slab is free once its previous store has read it out
        if (issuer) bulk_wait_read_all();
        if (!epi_sync()) break;
      }
      if (!mbar_wait(&acc_full[acc], aph, abort_flag)) break;
      if (AUX == AUX_LOAD && !mbar_wait(aux_full, it & 1, abort_flag)) break;
      tc_fence_after();
      const TileCoord tc = tile_coord(t, m_pairs, n_tiles, group_m);
      const int m_tile = 2 * tc.m + static_cast<int>(rank);
      Epi e = epi;
      e.begin_tile(m_tile, tc.n, row, q, lane, AUX == AUX_NONE ? nullptr : s_aux);
      e.begin_half(h);
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * TILE_N);
      // the 4 chunks of the half, with the TMEM load of chunk i + 1 in flight
      // while chunk i is processed
      uint32_t r0[32], r1[32];
      tmem_ld32_issue(t_row + c_begin, r0);
      tmem_ld32_wait(r0);
#pragma unroll
      for (int i = 0; i < (TILE_N / 2) / 32; ++i) {
        const int c = c_begin + 32 * i;
        uint32_t(&cur)[32] = (i & 1) ? r1 : r0;
        uint32_t(&nxt)[32] = (i & 1) ? r0 : r1;
        if (i + 1 < (TILE_N / 2) / 32) {
          tmem_ld32_issue(t_row + c + 32, nxt);
        } else {
          // every load of this accumulator has completed: the MMA warp may reuse it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(acc ? leader_acc_empty1 : leader_acc_empty0);
        }
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(cur[j]);
        e.chunk(c, v);
        if (i + 1 < (TILE_N / 2) / 32) tmem_ld32_wait(nxt);
      }
      e.end_half(h);
      if (AUX == AUX_LOAD) {
        __syncwarp();
        if (lane == 0) mbar_arrive(aux_empty);
      }
      e.end_tile();
      if (AUX == AUX_STORE) {
        fence_proxy_async_smem();
        if (!epi_sync()) break;
        if (issuer)
          aux_store_rows<Epi>(s_aux, &tm_aux, m_tile * TILE_M, tc.n * TILE_N, c_begin,
                              TILE_N / 2);
      }
    }
    if (AUX == AUX_STORE && issuer) bulk_wait_all();
  }

  // Teardown: the leader's MMAs write into both CTAs' TMEM, so neither CTA
  // frees TMEM before both have finished (bounded handshake on done_bar).
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) {
      mbar_arrive_remote(mapa_shared(smem_u32(done_bar), peer));
      mbar_wait_cluster(done_bar, 0, nullptr);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TC_TMEM_COLS);
  }
}

// CUDA-core version of the same tile: one thread per feature row, 32 token
// columns per pass, operands staged through shared memory in 32-wide K slabs.
// T may be any of bf16 / fp32 through the loader functor below.
constexpr int SIMT_K = 32;

template <class Epi>
__global__ void __launch_bounds__(TILE_M)
    simt_tile_gemm(const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ tok,
                   int n_rows, int n_cols, int k_dim, const Epi epi) {
  __shared__ float s_w[TILE_M][SIMT_K + 1];
  __shared__ float s_t[32][SIMT_K + 1];
  const int m_tile = blockIdx.y, n_tile = blockIdx.x;
  const int row = threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int q = threadIdx.x >> 5;
  const int f = m_tile * TILE_M + row;

  Epi e = epi;
  e.begin_tile(m_tile, n_tile, row, q, lane, nullptr);
  for (int c = 0; c < TILE_N; c += 32) {
    if (c % (TILE_N / 2) == 0) e.begin_half(c / (TILE_N / 2));
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.f;
    for (int k0 = 0; k0 < k_dim; k0 += SIMT_K) {
      __syncthreads();
      for (int i = threadIdx.x; i < TILE_M * SIMT_K; i += TILE_M) {
        const int r = i / SIMT_K, kk = i % SIMT_K;
        const int gf = m_tile * TILE_M + r, gk = k0 + kk;
        s_w[r][kk] = (gf < n_rows && gk < k_dim)
                         ? __bfloat162float(w[static_cast<size_t>(gf) * k_dim + gk])
                         : 0.f;
      }
      for (int i = threadIdx.x; i < 32 * SIMT_K; i += TILE_M) {
        const int r = i / SIMT_K, kk = i % SIMT_K;
        const int gt = n_tile * TILE_N + c + r, gk = k0 + kk;
        s_t[r][kk] = (gt < n_cols && gk < k_dim)
                         ? __bfloat162float(tok[static_cast<size_t>(gt) * k_dim + gk])
                         : 0.f;
      }
      __syncthreads();
#pragma unroll 4
      for (int kk = 0; kk < SIMT_K; ++kk) {
        const float a = s_w[row][kk];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaf(a, s_t[j][kk], v[j]);
      }
    }
    (void)f;
    e.chunk(c, v);
    if (c % (TILE_N / 2) == TILE_N / 2 - 32) e.end_half(c / (TILE_N / 2));
  }
  e.end_tile();
}

}  // namespace sae
