// NVLink peer-memory exchange of the dictionary-sharded forward.
//
// Every rank's peer buffer (its step workspace, then the exchange region, then
// the flags) is mapped into every other rank's address space (CUDA IPC). The
// forward's cross-shard sum becomes: each rank writes its fp32 decoder partial
// and per-token counts to its own exchange region; a flag barrier; rank r sums
// the partials of tokens [rB/N, (r+1)B/N) over all ranks with peer loads, in
// rank order, forms the residual, loss terms and go for those tokens and
// stores them straight into every rank's workspace with peer stores; a second
// flag barrier. The reduction and the residual run in one kernel, and the
// bytes crossing NVLink per rank are (N-1)/N * B * d * (4 + 2): the fp32
// partials read once and the bf16 go written once, against 8 per element for
// an all-reduce of the fp32 partials.
//
// Waits are bounded by wall-clock time: a barrier that runs out records
// SAE_ERR_DEVICE_TIMEOUT in the device status word and returns.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include "ptx.cuh"

namespace sae {

struct PeerArgs {
  char* base[SAE_MAX_PEERS];   // each rank's peer buffer in this process's address space
  int rank, world;
  uint32_t epoch;
  uint64_t exchange_off, flags_off;
  uint64_t go_off, tok_sqerr_off, tok_cnt_off, gosum_off;   // workspace regions
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Flag barrier across the ranks (one block, one thread per peer): post this
// rank's epoch into every peer's slot [phase][rank], then wait until every
// peer has posted it into ours. Epochs grow by one per use; the comparison is
// wrap-safe.
__global__ void peer_barrier_kernel(PeerArgs a, int phase) {
  const int p = threadIdx.x;
  const bool other = p < a.world && p != a.rank;
  if (other) {
    __threadfence_system();   // this rank's earlier writes before the flag
    uint32_t* slot = reinterpret_cast<uint32_t*>(a.base[p] + a.flags_off) +
                     phase * SAE_MAX_PEERS + a.rank;
    st_release_sys(slot, a.epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(a.base[a.rank] + a.flags_off) +
                           phase * SAE_MAX_PEERS + p;
    const uint64_t t0 = globaltimer_ns();
    while (static_cast<int32_t>(ld_acquire_sys(mine) - a.epoch) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_device_status(SAE_ERR_DEVICE_TIMEOUT);
        return;
      }
    }
  }
}

// Rank r's share of the exchange: tokens [lo, hi), block per token
// (grid-stride), d/8 threads. Sums the ranks' partials in rank order, then the
// residual of decode_kernel (x_hat = bf16(sum) + b_dec, r = x - x_hat,
// go = -(scale 2r) in bf16), and writes go, the token's squared error and
// active count into every rank's workspace. The block's running go sums go to
// row r * gridDim.x + blockIdx.x of every rank's go-sum partials.
template <typename XT>
__global__ void __launch_bounds__(1024)
    exchange_reduce_kernel(PeerArgs a, const XT* __restrict__ x, const float* __restrict__ b_dec,
                           int64_t n_tokens, int d, float go_scale, int64_t lo, int64_t hi) {
  __shared__ float s_tmp[33];
  const int col = threadIdx.x;
  const int nvec = d / 8;
  const bool has = col < nvec;
  float gsum[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) gsum[j] = 0.f;
  for (int64_t b = lo + blockIdx.x; b < hi; b += gridDim.x) {
    const size_t base = static_cast<size_t>(b) * d + col * 8;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    float cnt = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const float* part = reinterpret_cast<const float*>(a.base[p] + a.exchange_off);
      if (has) {
        const float4 u = *reinterpret_cast<const float4*>(part + base);
        const float4 v = *reinterpret_cast<const float4*>(part + base + 4);
        acc[0] += u.x; acc[1] += u.y; acc[2] += u.z; acc[3] += u.w;
        acc[4] += v.x; acc[5] += v.y; acc[6] += v.z; acc[7] += v.w;
      }
      if (col == 0) cnt += part[n_tokens * d + b];
    }
    float sq = 0.f;
    if (has) {
      float xv[8];
      if constexpr (sizeof(XT) == 2) {
        unpack8(*reinterpret_cast<const uint4*>(x + base), xv);
      } else {
        const float4 u = *reinterpret_cast<const float4*>(x + base);
        const float4 v = *reinterpret_cast<const float4*>(x + base + 4);
        xv[0] = u.x; xv[1] = u.y; xv[2] = u.z; xv[3] = u.w;
        xv[4] = v.x; xv[5] = v.y; xv[6] = v.z; xv[7] = v.w;
      }
      float gv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = __fadd_rn(bf16_round(acc[j]), b_dec[col * 8 + j]);
        const float r = __fsub_rn(xv[j], xh);
        sq = fmaf(r, r, sq);
        gv[j] = -__fmul_rn(go_scale, __fadd_rn(r, r));
        gsum[j] += gv[j];
      }
      const uint4 packed = pack8(gv);
      for (int p = 0; p < a.world; ++p)
        *reinterpret_cast<uint4*>(a.base[p] + a.go_off + base * 2) = packed;
    }
    const float tot = block_sum(sq, s_tmp);
    if (col == 0) {
      for (int p = 0; p < a.world; ++p) {
        reinterpret_cast<float*>(a.base[p] + a.tok_sqerr_off)[b] = tot;
        reinterpret_cast<int*>(a.base[p] + a.tok_cnt_off)[b] = static_cast<int>(cnt);
      }
    }
  }
  if (has) {
    const size_t row = static_cast<size_t>(a.rank) * gridDim.x + blockIdx.x;
    for (int p = 0; p < a.world; ++p) {
      float* g = reinterpret_cast<float*>(a.base[p] + a.gosum_off) + row * d + col * 8;
      reinterpret_cast<float4*>(g)[0] = make_float4(gsum[0], gsum[1], gsum[2], gsum[3]);
      reinterpret_cast<float4*>(g)[1] = make_float4(gsum[4], gsum[5], gsum[6], gsum[7]);
    }
  }
  __threadfence_system();   // peer stores performed before the next barrier's flag
}

}  // namespace sae
