// Dead-feature aux loss of the training step (sae_trainer_rolling.py:2986-2998):
//   pre_dead = relu(pre[:, dead]); (vals, idx) = topk(pre_dead, k) per token;
//   x_aux = bf16(Σ vals · W_dec[:, dead[idx]]); aux = coeff · mean((r - x_aux)^2) / accum
// with r = x - x_hat detached. Zero and negative pre-activations contribute
// nothing (relu), so only the positive candidates are ever selected.
//
// Layout: the selected entries of token b sit at [b * k, b * k + cnt[b]) of
// two arrays (dead-list index j, value), in increasing j; the backward sorts
// them by j (stable, so tokens ascend within a feature) and runs the sampled
// backward's kernel over that feature-major CSR.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include "ptx.cuh"

namespace sae {

constexpr int AUX_TB = 32;   // tokens per selection block (one per lane)
constexpr int AUX_DECODE_STAGE = 256;   // selected entries staged per pass

// bf16 bits of a positive value order like the value; everything else -> 0.
__device__ __forceinline__ uint32_t aux_key(uint16_t bits) {
  return (bits & 0x8000u) ? 0u : bits;
}

// Per block of 32 tokens: a two-pass radix select (high byte, then low byte
// of the bf16 key) finds each token's k-th largest positive key T and how
// many of the keys equal to T to take (the lowest dead indices first); a
// third pass over the dead rows writes the selected entries in dead order.
// 256 threads; rows are read as 64-byte segments of the feature-major
// pre-activations (one row = one dead feature's 32 tokens), 8 rows in flight
// per warp (16 without PACKED). PACKED (fewer than 65536 dead features): two 16-bit bin counts
// per 32-bit word, so the histograms take 16.5 KB and every block of a
// 32768-token step is resident at once (one wave).
template <bool PACKED>
struct AuxHist {
  static constexpr int kWords = PACKED ? 129 : 257;
  uint32_t w[AUX_TB][kWords];
  __device__ __forceinline__ void add(int t, uint32_t bin) {
    if constexpr (PACKED) atomicAdd(&w[t][bin >> 1], 1u << ((bin & 1u) * 16));
    else atomicAdd(&w[t][bin], 1u);
  }
  __device__ __forceinline__ uint32_t get(int t, int bin) const {
    if constexpr (PACKED) return (w[t][bin >> 1] >> ((bin & 1) * 16)) & 0xFFFFu;
    else return w[t][bin];
  }
};

template <bool PACKED>
__global__ void __launch_bounds__(256, PACKED ? 7 : 4)
    aux_select_kernel(const bf16* __restrict__ pre, int ldp, const int32_t* __restrict__ dead,
                      int n_dead, int n_features, int k, int64_t n_tokens,
                      int32_t* __restrict__ list_j,
                      float* __restrict__ list_v, int32_t* __restrict__ cnt,
                      int32_t* __restrict__ count_j) {
  constexpr int RW = PACKED ? 8 : 16;   // rows in flight per warp in the histogram passes
  __shared__ AuxHist<PACKED> hist;
  __shared__ uint16_t tile[32][AUX_TB + 2];
  __shared__ uint32_t s_hi[AUX_TB], s_above[AUX_TB], s_T[AUX_TB], s_m[AUX_TB];
  __shared__ int s_base[AUX_TB], s_ties[AUX_TB];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * AUX_TB;
  const bool tok_ok = t0 + lane < n_tokens;
  const uint16_t* pre16 = reinterpret_cast<const uint16_t*>(pre);
  uint32_t* hw = &hist.w[0][0];
  constexpr int HW = AUX_TB * AuxHist<PACKED>::kWords;

  auto key_at = [&](int j) -> uint32_t {
    if (!tok_ok) return 0u;
    const int f = min(max(dead[j], 0), n_features - 1);   // ids are checked by the caller
    return aux_key(pre16[static_cast<size_t>(f) * ldp + t0 + lane]);
  };

  // pass 1: histogram of the high byte of every positive key
  for (int i = tid; i < HW; i += blockDim.x) hw[i] = 0u;
  __syncthreads();
  for (int j0 = warp * RW; j0 < n_dead; j0 += 8 * RW) {
    uint32_t key[RW];
#pragma unroll
    for (int u = 0; u < RW; ++u) key[u] = j0 + u < n_dead ? key_at(j0 + u) : 0u;
#pragma unroll
    for (int u = 0; u < RW; ++u)
      if (key[u]) hist.add(lane, key[u] >> 8);
  }
  __syncthreads();
  if (tid < AUX_TB) {
    uint32_t cum = 0, hi = 0, total = 0;
    for (int b = 255; b >= 0; --b) total += hist.get(tid, b);
    if (total <= static_cast<uint32_t>(k)) {
      s_hi[tid] = 0xFFFFFFFFu;   // take every positive key
      s_above[tid] = 0;
    } else {
      for (int b = 255; b >= 0; --b) {
        const uint32_t h = hist.get(tid, b);
        if (cum + h >= static_cast<uint32_t>(k)) {
          hi = b;
          break;
        }
        cum += h;
      }
      s_hi[tid] = hi;
      s_above[tid] = cum;
    }
  }
  __syncthreads();
  // pass 2: low byte inside the chosen high-byte bin
  for (int i = tid; i < HW; i += blockDim.x) hw[i] = 0u;
  __syncthreads();
  {
    const uint32_t hi = s_hi[lane];
    for (int j0 = warp * RW; j0 < n_dead; j0 += 8 * RW) {
      uint32_t key[RW];
#pragma unroll
      for (int u = 0; u < RW; ++u) key[u] = j0 + u < n_dead ? key_at(j0 + u) : 0u;
#pragma unroll
      for (int u = 0; u < RW; ++u)
        if (key[u] && (key[u] >> 8) == hi) hist.add(lane, key[u] & 0xFFu);
    }
  }
  __syncthreads();
  if (tid < AUX_TB) {
    if (s_hi[tid] == 0xFFFFFFFFu) {
      s_T[tid] = 1u;              // every positive key is > 0
      s_m[tid] = 0xFFFFFFFFu;
    } else {
      uint32_t cum = s_above[tid];
      uint32_t lo = 0;
      for (int b = 255; b >= 0; --b) {
        const uint32_t h = hist.get(tid, b);
        if (cum + h >= static_cast<uint32_t>(k)) {
          lo = b;
          break;
        }
        cum += h;
      }
      s_T[tid] = (s_hi[tid] << 8) | lo;
      s_m[tid] = static_cast<uint32_t>(k) - cum;   // keys equal to T still to take
    }
    s_base[tid] = 0;
    s_ties[tid] = 0;
  }
  // pass 3: rows in chunks of 32 through shared memory; warp w loads rows
  // w, w + 8, w + 16, w + 24 of the next chunk while the current one is
  // scanned, owns tokens w, w + 8, w + 16, w + 24 and walks the chunk's rows
  // in order (lane = row)
  uint32_t nxt[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) nxt[q] = (8 * q + warp < n_dead) ? key_at(8 * q + warp) : 0u;
  for (int j0 = 0; j0 < n_dead; j0 += 32) {
    __syncthreads();   // the previous chunk's tile is consumed (and pass 2's state is set)
#pragma unroll
    for (int q = 0; q < 4; ++q) tile[8 * q + warp][lane] = static_cast<uint16_t>(nxt[q]);
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int j = j0 + 32 + 8 * q + warp;
      nxt[q] = j < n_dead ? key_at(j) : 0u;
    }
    const uint32_t lt = (1u << lane) - 1u;
    for (int q = warp; q < AUX_TB; q += 8) {
      const int64_t b = t0 + q;
      if (b >= n_tokens) continue;   // uniform per warp
      const int j = j0 + lane;
      const uint32_t key = (j < n_dead) ? tile[lane][q] : 0u;
      const uint32_t T = s_T[q];
      const bool eq = key != 0u && key == T;
      const uint32_t eqb = __ballot_sync(0xffffffffu, eq);
      const uint32_t rank = static_cast<uint32_t>(s_ties[q]) + __popc(eqb & lt);
      const bool sel = key != 0u && (key > T || (eq && rank < s_m[q]));
      const uint32_t sb = __ballot_sync(0xffffffffu, sel);
      const int pos = s_base[q] + __popc(sb & lt);
      if (sel && pos < k) {
        list_j[b * k + pos] = j;
        list_v[b * k + pos] = __uint_as_float(key << 16);
        atomicAdd(&count_j[j], 1);
      }
      __syncwarp();
      if (lane == 0) {
        s_base[q] += __popc(sb);
        s_ties[q] += __popc(eqb);
      }
      __syncwarp();
    }
  }
  __syncthreads();
  if (tid < AUX_TB && t0 + tid < n_tokens) cnt[t0 + tid] = min(s_base[tid], k);
}

// Per token (grid-stride, d/8 threads): x_aux = bf16(Σ v · W_dec[dead[j]])
// over the token's selected entries in dead order, e = (x - x_hat) - x_aux,
// the token's Σ e² and g = bf16(-(2 coeff / (B d accum)) e), the gradient
// reaching x_aux (what the bf16 aux matmul's backward sees).
template <typename XT>
__global__ void __launch_bounds__(1024)
    aux_decode_kernel(const int32_t* __restrict__ list_j, const float* __restrict__ list_v,
                      const int32_t* __restrict__ cnt, const int32_t* __restrict__ dead,
                      int n_features, int k,
                      const bf16* __restrict__ w_dec, const XT* __restrict__ x,
                      const float* __restrict__ x_hat, int64_t n_tokens, int d, float g_scale,
                      bf16* __restrict__ g_aux, float* __restrict__ aux_sq) {
  // The token's selected entries (decoder row, value) are staged in shared
  // memory by one load per thread, then the rows are gathered eight at a
  // time; the sum runs over the entries in list order, as before staging.
  __shared__ float s_tmp[33];
  __shared__ int s_f[AUX_DECODE_STAGE];
  __shared__ float s_a[AUX_DECODE_STAGE];
  const int col = threadIdx.x;
  const int nvec = d / 8;
  const bool has = col < nvec;
  const uint4* wcol = reinterpret_cast<const uint4*>(w_dec) + col;
  for (int64_t b = blockIdx.x; b < n_tokens; b += gridDim.x) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    const int n = cnt[b];
    float sq = 0.f;
    for (int w0 = 0; w0 < n; w0 += AUX_DECODE_STAGE) {
      const int m = min(AUX_DECODE_STAGE, n - w0);
      __syncthreads();   // the previous window's entries are consumed
      for (int e = threadIdx.x; e < m; e += blockDim.x) {
        const size_t li = static_cast<size_t>(b) * k + w0 + e;
        s_f[e] = min(max(dead[list_j[li]], 0), n_features - 1);
        s_a[e] = list_v[li];
      }
      __syncthreads();
      if (has) {
        int i = 0;
        for (; i + 7 < m; i += 8) {
          uint4 u[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) u[r] = __ldg(wcol + static_cast<size_t>(s_f[i + r]) * nvec);
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            float wf[8];
            unpack8(u[r], wf);
            const float a = s_a[i + r];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(a, wf[j], acc[j]);
          }
        }
        for (; i < m; ++i) {
          float wf[8];
          unpack8(__ldg(wcol + static_cast<size_t>(s_f[i]) * nvec), wf);
          const float a = s_a[i];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = fmaf(a, wf[j], acc[j]);
        }
      }
    }
    if (has) {
      const size_t base = static_cast<size_t>(b) * d + col * 8;
      float xv[8];
      if constexpr (sizeof(XT) == 2) {
        unpack8(*reinterpret_cast<const uint4*>(x + base), xv);
      } else {
        const float4 a = *reinterpret_cast<const float4*>(x + base);
        const float4 c = *reinterpret_cast<const float4*>(x + base + 4);
        xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
        xv[4] = c.x; xv[5] = c.y; xv[6] = c.z; xv[7] = c.w;
      }
      const float4 h0 = *reinterpret_cast<const float4*>(x_hat + base);
      const float4 h1 = *reinterpret_cast<const float4*>(x_hat + base + 4);
      const float xh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
      float gv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float r = __fsub_rn(xv[j], xh[j]);
        const float e = __fsub_rn(r, bf16_round(acc[j]));
        sq = fmaf(e, e, sq);
        gv[j] = -__fmul_rn(g_scale, e);
      }
      *reinterpret_cast<uint4*>(g_aux + base) = pack8(gv);
    }
    const float tot = block_sum(sq, s_tmp);
    if (threadIdx.x == 0) aux_sq[b] = tot;
  }
}

// aux = coeff * Σ_b aux_sq[b] / (B d) / accum, added to the step's loss.
__global__ void __launch_bounds__(1024)
    aux_stats_kernel(const float* __restrict__ aux_sq, int64_t n_tokens, int d, float coeff,
                     int accum, SaeB200StepStats* stats) {
  __shared__ float s_tmp[33];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n_tokens; i += blockDim.x) s += aux_sq[i];
  const float tot = block_sum(s, s_tmp);
  if (threadIdx.x == 0) {
    const float aux = tot / static_cast<float>(static_cast<double>(n_tokens) * d) * coeff /
                      static_cast<float>(accum);
    stats->aux_loss = aux;
    stats->loss += aux;
  }
}

// Sort keys/values for the backward: key = dead-list index (n_dead for an
// empty slot, sorted last), value = token << 32 | float bits of the value.
__global__ void aux_pack_kernel(const int32_t* __restrict__ list_j,
                                const float* __restrict__ list_v, const int32_t* __restrict__ cnt,
                                int64_t n_tokens, int k, int n_dead, uint32_t* __restrict__ keys,
                                uint64_t* __restrict__ vals) {
  const int64_t total = n_tokens * k;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = i / k;
    const int r = static_cast<int>(i - b * k);
    const bool ok = r < cnt[b];
    keys[i] = ok ? static_cast<uint32_t>(list_j[i]) : static_cast<uint32_t>(n_dead);
    vals[i] = ok ? ((static_cast<uint64_t>(b) << 32) | __float_as_uint(list_v[i])) : 0ull;
  }
}

// Sorted aux entries -> the sampled backward's CSR format: token, and the
// bf16 value (exact: it is a relu'd bf16 pre-activation) flagged active.
__global__ void aux_unpack_kernel(const uint64_t* __restrict__ vals, const int32_t* __restrict__ offs,
                                  int n_dead, int* __restrict__ csr_tok,
                                  uint32_t* __restrict__ csr_val) {
  const int total = offs[n_dead];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint64_t v = vals[i];
    csr_tok[i] = static_cast<int>(v >> 32);
    csr_val[i] = (static_cast<uint32_t>(v) >> 16) | CSR_ACTIVE;
  }
}

}  // namespace sae
