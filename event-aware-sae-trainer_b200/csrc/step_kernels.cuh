// Kernels of one fused JumpReLU SAE training step (forward, backward,
// gradient norm, Adam + renormalisation). The launch order and the buffers
// they share are set up in capi.cu.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include "ptx.cuh"
#include "tile_gemm.cuh"

namespace sae {

using bf16 = __nv_bfloat16;

// Fixed grid sizes: partial sums are reduced in a fixed order, so a given
// input produces bit-identical results on every run and every B200.
constexpr int DECODE_GRID = 2368;   // 148 SMs x 16 (blocks of a few tokens: short tails)
constexpr int GEMV_GRID = 1184;
constexpr int NORM_GRID = SAE_GRAD_NORM_WORKSPACE_BYTES / 4;
constexpr int DECODE_LIST_CAP = 2048;   // active features staged per pass

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ void unpack8(const uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Two independent fp32 FMAs in one instruction (sm_100 fma.rn.f32x2):
// (d0, d1) = (a0 * b0 + d0, a1 * b1 + d1), each rounded like fmaf.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0,
                                     float b1) {
  uint64_t d, a, b;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(d0), "f"(d1));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return l | (h << 16);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack2(f[0], f[1]);
  u.y = pack2(f[2], f[3]);
  u.z = pack2(f[4], f[5]);
  u.w = pack2(f[6], f[7]);
  return u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum in a fixed order; result valid in every thread.
__device__ __forceinline__ float block_sum(float v, float* s_tmp) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) s_tmp[wid] = v;
  __syncthreads();
  float t = 0.f;
  if (wid == 0) {
    t = lane < nw ? s_tmp[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) s_tmp[32] = t;
  }
  __syncthreads();
  return s_tmp[32];
}

// Block-wide exclusive scan of ints; also returns the block total.
__device__ __forceinline__ int block_excl_scan(int v, int* s_tmp, int& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) s_tmp[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int t = lane < nw ? s_tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    s_tmp[lane] = t;   // inclusive prefix of warp totals
  }
  __syncthreads();
  total = s_tmp[nw - 1];
  return (wid > 0 ? s_tmp[wid - 1] : 0) + x - v;
}

// ---------------------------------------------------------------- prologue
// theta = exp(log_threshold) (the same expf the reference's CUDA exp uses),
// xc = bf16(float(x) - b_dec): autocast's cast of the fp32 difference
// (sae_trainer_rolling.py:586-588).
// ------------------------------------------------- gate cut values
// For a feature with threshold th and bf16-rounded bias b, the encoder gate of
// an accumulator v is [bf16(v + b) > th] and its sampled-backward entry bit is
// [bf16(v + b) - th > -eps] (fp32 add and subtract, round to nearest). Each
// step rounds monotonically, so each predicate is [v >= cut] for the least
// float cut that satisfies it. gate_cut finds cut by bisection over the
// ordered float keys, evaluating the predicate with exactly those operations;
// the encoder epilogue then reads each bit off the sign of fl(v - cut), which
// is exact: a nonzero difference never rounds to zero, and v = cut gives +0.
// A zero cut is returned as -0, so that fl(v + 0) keeps v's sign for v = -0.
__device__ __forceinline__ uint32_t float_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
template <bool ENTRY>
__device__ float gate_cut(float bias, float th, float neg_eps) {
  auto pass = [&](float v) {
    const float p = bf16_round(__fadd_rn(v, bias));
    return ENTRY ? (__fsub_rn(p, th) > neg_eps) : (p > th);
  };
  const float inf = __int_as_float(0x7F800000);
  if (!pass(inf)) return inf;     // no finite v passes
  if (pass(-inf)) return -inf;    // every finite v passes
  uint32_t lo = float_key(-inf), hi = float_key(inf);   // pass(lo) false, pass(hi) true
  while (hi - lo > 1u) {
    const uint32_t mid = lo + (hi - lo) / 2u;
    if (pass(key_float(mid))) hi = mid;
    else lo = mid;
  }
  const float c = key_float(hi);
  return c == 0.f ? -0.f : c;
}

// theta = exp(log_threshold) and, when cut is set, each feature's gate cut
// values (x: active, y: sampled-backward entry at bandwidth eps); xc = x - b_dec
// in bf16.
template <typename XT>
__global__ void prep_kernel(const XT* __restrict__ x, const float* __restrict__ b_dec,
                            const float* __restrict__ log_thr, const float* __restrict__ b_enc,
                            float eps, float* __restrict__ theta, float2* __restrict__ cut,
                            bf16* __restrict__ xc, int64_t n_tokens, int d, int n_features) {
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t f = tid; f < n_features; f += stride) {
    const float th = expf(log_thr[f]);
    theta[f] = th;
    if (cut != nullptr) {
      const float b = bf16_round(b_enc[f]);
      cut[f] = make_float2(gate_cut<false>(b, th, -eps), gate_cut<true>(b, th, -eps));
    }
  }
  const int64_t nvec = n_tokens * (d / 8);
  const int dv = d / 8;
  auto one = [&](int64_t i, const float (&xv)[8]) {
    const int c = static_cast<int>(i % dv) * 8;
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __fsub_rn(xv[j], b_dec[c + j]);
    reinterpret_cast<uint4*>(xc)[i] = pack8(r);
  };
  auto load = [&](int64_t i, float (&xv)[8]) {
    if constexpr (sizeof(XT) == 2) {
      unpack8(reinterpret_cast<const uint4*>(x)[i], xv);
    } else {
      const float4 a = reinterpret_cast<const float4*>(x)[2 * i];
      const float4 b = reinterpret_cast<const float4*>(x)[2 * i + 1];
      xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
      xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
    }
  };
  // four vectors per thread in flight
  int64_t i = tid;
  for (; i + 3 * stride < nvec; i += 4 * stride) {
    float xv[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) load(i + u * stride, xv[u]);
#pragma unroll
    for (int u = 0; u < 4; ++u) one(i + u * stride, xv[u]);
  }
  for (; i < nvec; i += stride) {
    float xv[8];
    load(i, xv);
    one(i, xv);
  }
}

// ------------------------------------------------- side-tile helpers
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The pre-activations of a microbatch are kept feature-major, [F, ldp] bf16
// (ldp = n_tokens rounded up to 64): the tile epilogues, where a thread owns
// one feature, then read and write 8 consecutive tokens per 16-byte access.

// -------------------------------------------------- encoder tile epilogue
// pre = bf16(acc + bf16(b_enc)) (cuBLAS addmm with a bf16 bias); gate bit =
// float(pre) > theta. Stores pre, one 32-feature mask word per token per
// warp, and the active-token count of each feature in each 128-token half of
// the tile (the unit the epilogue warps split a tile into).
// What the encoder epilogue stores of pre:
//   PRE_FULL     every element, through the side tile's TMA store (the dense
//                backward and the aux loss read all of it)
//   PRE_ENTRIES  only the 32-token words of a feature that hold an active or
//                in-band entry (direct 64-byte stores): the decode reads pre
//                at the active entries and the CSR fill at the sampled-
//                backward entries, nothing else reads it. Of the d=1536,
//                F=49152, L0~50 step's 3.2 GB of pre, a few percent is stored.
constexpr int PRE_FULL = 0;
constexpr int PRE_ENTRIES = 1;

template <int PRE>
struct EncodeEpiT {
  static constexpr int kAux = PRE == PRE_FULL ? AUX_STORE : AUX_NONE;
  static constexpr bool kAuxFeatureMajor = true;
  const float2* cut;   // per feature: gate cut values (active, entry) of gate_cut
  const float* b_enc;
  bf16* pre;          // [F, ldp]
  uint32_t* mask;
  int* tile_cnt;
  // Sampled backward (optional): its entries are the (token, feature) pairs with
  // pre - theta > -eps, i.e. active (pre > theta) or inside the STE band
  // |pre - theta| < eps. sbits [ldp / 32, F] holds one bit each (word w of
  // feature f: tokens 32w..32w+31), so that the 32 features of an epilogue warp
  // store one coalesced line.
  uint32_t* sbits;
  // per-feature totals (optional): with act_sum set, each half tile's counts
  // are added to act_sum[f] / entry_sum[f] instead of stored per tile
  int* act_sum;
  int* entry_sum;
  int n_tokens, n_features, mask_words, ldp;
  // per-thread tile state
  int f, n0, lane, word, row;
  float neg_cut_a, neg_cut_s, bias;
  int cnt, bcnt;
  bool row_ok;
  bf16* aux;

  __device__ __forceinline__ void begin_tile(int m_tile, int n_tile, int r, int q, int ln,
                                             bf16* aux_tile) {
    row = r;
    f = m_tile * TILE_M + r;
    n0 = n_tile * TILE_N;
    lane = ln;
    aux = aux_tile;
    row_ok = f < n_features;
    const float2 ct = row_ok ? cut[f] : make_float2(__int_as_float(0x7f800000),
                                                    __int_as_float(0x7f800000));
    neg_cut_a = -ct.x;
    neg_cut_s = -ct.y;
    bias = row_ok ? bf16_round(b_enc[f]) : 0.f;
    word = (m_tile * TILE_M + q * 32) >> 5;
  }
  __device__ __forceinline__ void begin_half(int) {
    cnt = 0;
    bcnt = 0;
  }
  __device__ __forceinline__ void chunk(int c, const float (&v)[32]) {
    const int t0 = n0 + c;
    const int nj = row_ok ? min(32, n_tokens - t0) : 0;
    const uint32_t valid = nj >= 32 ? 0xFFFFFFFFu : (nj <= 0 ? 0u : (1u << nj) - 1u);
    // aw: this feature's gate bits over the chunk's 32 tokens; sword: its
    // sampled-backward entries (active or in band). Bit j is set where
    // v[j] >= cut, i.e. where fl(v[j] - cut) has its sign bit clear; the sign
    // bits are shifted in from token 15 (31) down, two chains per mask.
    uint32_t na0 = 0u, na1 = 0u, ns0 = 0u, ns1 = 0u;
#pragma unroll
    for (int k = 7; k >= 0; --k) {
      const float2 lo = make_float2(v[2 * k], v[2 * k + 1]);
      const float2 hi = make_float2(v[16 + 2 * k], v[17 + 2 * k]);
      const float2 la = __fadd2_rn(lo, make_float2(neg_cut_a, neg_cut_a));
      const float2 ha = __fadd2_rn(hi, make_float2(neg_cut_a, neg_cut_a));
      const float2 ls = __fadd2_rn(lo, make_float2(neg_cut_s, neg_cut_s));
      const float2 hs = __fadd2_rn(hi, make_float2(neg_cut_s, neg_cut_s));
      na0 = __funnelshift_l(__float_as_uint(la.y), na0, 1);
      na0 = __funnelshift_l(__float_as_uint(la.x), na0, 1);
      na1 = __funnelshift_l(__float_as_uint(ha.y), na1, 1);
      na1 = __funnelshift_l(__float_as_uint(ha.x), na1, 1);
      ns0 = __funnelshift_l(__float_as_uint(ls.y), ns0, 1);
      ns0 = __funnelshift_l(__float_as_uint(ls.x), ns0, 1);
      ns1 = __funnelshift_l(__float_as_uint(hs.y), ns1, 1);
      ns1 = __funnelshift_l(__float_as_uint(hs.x), ns1, 1);
    }
    const uint32_t aw = ~((na1 << 16) | na0) & valid;
    const uint32_t sword = ~((ns1 << 16) | ns0) & valid;
    // the bf16 pre-activations, where they are stored
    auto pack_pre = [&](uint32_t (&pk)[16]) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 s = __fadd2_rn(make_float2(v[2 * i], v[2 * i + 1]), make_float2(bias, bias));
        pk[i] = pack_bf2(s.x, s.y);
      }
    };
    cnt += __popc(aw);
    // 32x32 bit transpose across the warp (lane = feature -> lane = token):
    // afterwards lane j holds the mask word of token t0 + j over the warp's
    // 32 features
    uint32_t myword = aw;
#pragma unroll
    for (int sh = 16; sh >= 1; sh >>= 1) {
      const uint32_t m = sh == 16 ? 0x0000FFFFu : sh == 8 ? 0x00FF00FFu
                       : sh == 4 ? 0x0F0F0F0Fu : sh == 2 ? 0x33333333u : 0x55555555u;
      const uint32_t y = __shfl_xor_sync(0xffffffffu, myword, sh);
      myword = (lane & sh) ? ((myword & ~m) | ((y >> sh) & m)) : ((myword & m) | ((y << sh) & ~m));
    }
    if (sbits != nullptr) {
      bcnt += __popc(sword);
      if (nj > 0) sbits[static_cast<size_t>(t0 >> 5) * n_features + f] = sword;
    }
    if (aux != nullptr) {
      // tokens past n_tokens are clipped by the TMA store
      uint32_t pk[16];
      pack_pre(pk);
      uint8_t* base = reinterpret_cast<uint8_t*>(aux);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(base + aux_fm_offset(row, (c >> 3) + q)) =
            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    } else if (row_ok && (PRE == PRE_FULL || (aw | sword) != 0u)) {
      uint32_t pk[16];
      pack_pre(pk);
      bf16* dst = pre + static_cast<size_t>(f) * ldp + t0;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (8 * q < nj)   // ldp is a multiple of 64: whole 8-token groups stay in the row
          *reinterpret_cast<uint4*>(dst + 8 * q) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    }
    const int t = t0 + lane;
    if (t < n_tokens && word < mask_words)
      mask[static_cast<size_t>(t) * mask_words + word] = myword;
  }
  __device__ __forceinline__ void end_half(int h) {
    if (!row_ok) return;
    if (act_sum != nullptr) {
      if (cnt != 0) atomicAdd(act_sum + f, cnt);
      if (bcnt != 0) atomicAdd(entry_sum + f, bcnt);
      return;
    }
    tile_cnt[static_cast<size_t>(n0 / HALF_N + h) * n_features + f] = cnt;
  }
  __device__ __forceinline__ void end_tile() {}
};
using EncodeEpi = EncodeEpiT<PRE_FULL>;

// pre only, token-major [B, F] (module API encode_pre in bf16 mode).
struct PreOnlyEpi {
  static constexpr int kAux = AUX_STORE;
  static constexpr bool kAuxFeatureMajor = false;
  const float* b_enc;
  bf16* pre;
  int n_tokens, n_features;
  int f, n0, row;
  float bias;
  bool row_ok;
  bf16* aux;
  __device__ __forceinline__ void begin_tile(int m_tile, int n_tile, int r, int, int,
                                             bf16* aux_tile) {
    row = r;
    f = m_tile * TILE_M + r;
    n0 = n_tile * TILE_N;
    aux = aux_tile;
    row_ok = f < n_features;
    bias = row_ok ? bf16_round(b_enc[f]) : 0.f;
  }
  __device__ __forceinline__ void begin_half(int) {}
  __device__ __forceinline__ void end_half(int) {}
  __device__ __forceinline__ void chunk(int c, const float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int t = n0 + c + j;
      const bf16 p = __float2bfloat16_rn(v[j] + bias);
      if (aux != nullptr)
        aux[(c + j) * TILE_M + row] = p;
      else if (row_ok && t < n_tokens)
        pre[static_cast<size_t>(t) * n_features + f] = p;
    }
  }
  __device__ __forceinline__ void end_tile() {}
};

// ------------------------------------------------- backward tile epilogue
// acc = go . W_dec[f] is the dense grad_feat (bf16 GEMM output in the
// reference, 643). Per (token, feature):
//   combined = pre * grad_feat + gate_grad                   (hook, 805-817)
//   STE sum  += combined   where |pre - theta| < eps          (818-825)
//   dpre      = grad_feat  where pre > theta                   (grad_pre, gated)
// The per-feature sums of each 128-token half go to thr_part / dbenc_part; active
// pairs are appended to the feature-major CSR (token, pre, dpre) at the
// positions the scan assigned, in token order.
struct GradEpi {
  static constexpr int kAux = AUX_LOAD;   // the pre tile arrives in shared memory by TMA
  static constexpr bool kAuxFeatureMajor = true;
  const float* theta;
  const bf16* pre;    // [F, ldp]
  const int* col_offs;
  const int* tile_base;
  const SaeB200StepStats* stats;
  float eps;
  int n_tokens, n_features, ldp;
  int* csr_tok;
  uint32_t* csr_val;
  float* thr_part;
  float* dbenc_part;
  bf16* dense_dpre;   // non-null: write the gated gradient densely ([F, ldp]) instead of the CSR
  // per-thread tile state
  int f, n0, pos, row;
  float th, gate_grad, thr_sum, db_sum;
  bool row_ok, write_csr;
  const bf16* aux;

  __device__ __forceinline__ void begin_tile(int m_tile, int n_tile, int r, int, int,
                                             const bf16* aux_tile) {
    row = r;
    aux = aux_tile;
    f = m_tile * TILE_M + r;
    n0 = n_tile * TILE_N;
    row_ok = f < n_features;
    th = row_ok ? theta[f] : 0.f;
    gate_grad = stats->gate_grad;
    write_csr = (dense_dpre == nullptr) && (stats->csr_overflow == 0);
  }
  __device__ __forceinline__ void begin_half(int h) {
    pos = (row_ok && write_csr)
              ? col_offs[f] + tile_base[static_cast<size_t>(n0 / HALF_N + h) * n_features + f]
              : 0;
    thr_sum = 0.f;
    db_sum = 0.f;
  }
  __device__ __forceinline__ void chunk(int c, const float (&v)[32]) {
    if (!row_ok) return;
    const int t0 = n0 + c;
    const int nj = min(32, n_tokens - t0);
    uint32_t pw[16];   // 32 bf16 pre-activations, two per word
    if (aux != nullptr) {
      const uint8_t* base = reinterpret_cast<const uint8_t*>(aux);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 u = *reinterpret_cast<const uint4*>(base + aux_fm_offset(row, (c >> 3) + q));
        pw[4 * q] = u.x;
        pw[4 * q + 1] = u.y;
        pw[4 * q + 2] = u.z;
        pw[4 * q + 3] = u.w;
      }
    } else {
      const bf16* src = pre + static_cast<size_t>(f) * ldp + t0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u = make_uint4(0, 0, 0, 0);
        if (8 * q < nj) u = *reinterpret_cast<const uint4*>(src + 8 * q);
        pw[4 * q] = u.x;
        pw[4 * q + 1] = u.y;
        pw[4 * q + 2] = u.z;
        pw[4 * q + 3] = u.w;
      }
    }
    const float2 gg = make_float2(gate_grad, gate_grad);
    uint32_t dw[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t gw = pack_bf2(v[2 * i], v[2 * i + 1]);   // grad_feat as bf16
      const float2 p = make_float2(bf_lo(pw[i]), bf_hi(pw[i]));
      const float2 g = make_float2(bf_lo(gw), bf_hi(gw));
      const float2 comb = __fadd2_rn(__fmul2_rn(p, g), gg);
      const int j = 2 * i;
      if (j < nj && fabsf(__fsub_rn(p.x, th)) < eps) thr_sum += comb.x;
      if (j + 1 < nj && fabsf(__fsub_rn(p.y, th)) < eps) thr_sum += comb.y;
      const bool a0 = (j < nj) && p.x > th;
      const bool a1 = (j + 1 < nj) && p.y > th;
      dw[i] = (a0 ? (gw & 0xFFFFu) : 0u) | (a1 ? (gw & 0xFFFF0000u) : 0u);
      if (a0 | a1) {   // rare: ~L0 / F of the entries
        if (a0) {
          db_sum += g.x;
          if (write_csr) {
            csr_tok[pos] = n0 + c + j;
            csr_val[pos] = (pw[i] & 0xFFFFu) | (gw << 16);
          }
          ++pos;
        }
        if (a1) {
          db_sum += g.y;
          if (write_csr) {
            csr_tok[pos] = n0 + c + j + 1;
            csr_val[pos] = (pw[i] >> 16) | (gw & 0xFFFF0000u);
          }
          ++pos;
        }
      }
    }
    if (dense_dpre != nullptr) {
      bf16* dst = dense_dpre + static_cast<size_t>(f) * ldp + t0;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (8 * q < nj)
          *reinterpret_cast<uint4*>(dst + 8 * q) =
              make_uint4(dw[4 * q], dw[4 * q + 1], dw[4 * q + 2], dw[4 * q + 3]);
    }
  }
  __device__ __forceinline__ void end_half(int h) {
    if (!row_ok) return;
    const size_t i = static_cast<size_t>(n0 / HALF_N + h) * n_features + f;
    thr_part[i] = thr_sum;
    dbenc_part[i] = db_sum;
  }
  __device__ __forceinline__ void end_tile() {}
};

// ------------------------------------------------------------------- scans
// Per feature: exclusive prefix of the per-tile active counts (in place),
// the feature's total, and the OR-accumulated fired flag (the GEMM backward
// and the inference forward; the sampled forward adds per-feature totals in
// the encoder epilogue instead).
__global__ void scan_columns_kernel(int* __restrict__ tile_cnt, int* __restrict__ col_tot,
                                    uint8_t* __restrict__ fired, int n_tiles, int n_features) {
  for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < n_features;
       f += gridDim.x * blockDim.x) {
    int run = 0;
    for (int t = 0; t < n_tiles; ++t) {
      const size_t i = static_cast<size_t>(t) * n_features + f;
      const int v = tile_cnt[i];
      tile_cnt[i] = run;
      run += v;
    }
    col_tot[f] = run;
    if (fired != nullptr && run > 0) fired[f] = 1;
  }
}

// After the CSR offset scan of the sampled forward (col_offs[F] = entries):
// nnz = sum of the per-feature active counts (fixed-order block reduction),
// the fired flags, csr_pairs and the overflow flag; resets the backward's
// feature counter.
__global__ void __launch_bounds__(1024)
    count_stats_kernel(const int* __restrict__ col_act, const int* __restrict__ col_offs,
                       int n_features, int64_t capacity, SaeB200StepStats* stats,
                       int* counters, uint8_t* __restrict__ fired) {
  __shared__ int s_tmp[33];
  int local = 0;
  // 8 independent loads in flight per thread (one block walks all features)
  for (int f0 = threadIdx.x; f0 < n_features; f0 += 8 * blockDim.x) {
    int a[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int f = f0 + u * blockDim.x;
      a[u] = f < n_features ? col_act[f] : 0;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      local += a[u];
      if (fired != nullptr && a[u] > 0) fired[f0 + u * blockDim.x] = 1;
    }
  }
  int total = 0;
  block_excl_scan(local, s_tmp, total);
  if (threadIdx.x == 0) {
    const int pairs = col_offs[n_features];
    stats->nnz = total;
    stats->csr_pairs = pairs;
    stats->csr_overflow = (static_cast<int64_t>(pairs) > capacity) ? 1 : 0;
    counters[0] = 0;
  }
}

// Exclusive scan of the per-feature totals into CSR row offsets (one block).
__global__ void __launch_bounds__(1024)
    scan_offsets_kernel(const int* __restrict__ col_tot, int* __restrict__ col_offs, int n_features,
                        int64_t capacity, SaeB200StepStats* stats, int* counters) {
  __shared__ int s_tmp[33];
  const int per = (n_features + blockDim.x - 1) / blockDim.x;
  const int b = threadIdx.x * per;
  const int e = min(n_features, b + per);
  int local = 0;
#pragma unroll 8
  for (int i = b; i < e; ++i) local += col_tot[i];
  int total = 0;
  int run = block_excl_scan(local, s_tmp, total);
#pragma unroll 8
  for (int i = b; i < e; ++i) {
    col_offs[i] = run;
    run += col_tot[i];
  }
  if (threadIdx.x == 0) {
    col_offs[n_features] = total;
    stats->nnz = total;   // every entry of this CSR is active
    stats->csr_pairs = total;
    stats->csr_overflow = (static_cast<int64_t>(total) > capacity) ? 1 : 0;
    counters[0] = 0;
  }
}

// ----------------------------------------------------- sampled backward
// The straight-through backward needs grad_feat = go . W_dec[f] only where
// it is used: on active entries (grad_pre, db_enc, dW_enc) and on entries
// inside the STE band |pre - theta| < eps (the threshold gradient); the rest of
// the dense [B, F] product is multiplied by zero. The sampled path builds a
// feature-major CSR of exactly those entries and computes each one as a dot
// product of two bf16 rows.
//
// CSR fill: the encoder epilogue left one bit per (feature, token) entry in
// sbits [ldp / 32, F]. A block of 8 warps takes 32 consecutive features; per
// 1024-token window it loads the [32 words x 32 features] bit tile with
// coalesced rows, and warp w then walks features 4w..4w+3 of it: lane l holds
// word l of the window, a warp scan places the entries in token order after the
// feature's running offset, and each entry's bf16 pre-activation is read back.
// Entry value: low 16 bits bf16 pre, bit 16 active (pre > theta), bit 17 in
// band (|pre - theta| < eps).
constexpr uint32_t CSR_ACTIVE = 1u << 16;
constexpr uint32_t CSR_BAND = 1u << 17;

__global__ void __launch_bounds__(256)
    csr_fill_kernel(const bf16* __restrict__ pre, const uint32_t* __restrict__ sbits,
                    const float* __restrict__ theta, const int* __restrict__ col_offs,
                    int n_features, int64_t n_tokens, int ldp, float eps,
                    const SaeB200StepStats* stats, int* __restrict__ csr_tok,
                    uint32_t* __restrict__ csr_val) {
  if (stats->csr_overflow) return;
  __shared__ uint32_t tile[32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_words = static_cast<int>((n_tokens + 31) >> 5);
  const uint16_t* pre16 = reinterpret_cast<const uint16_t*>(pre);
  for (int f0 = blockIdx.x * 32; f0 < n_features; f0 += gridDim.x * 32) {
    int pos[4], end[4];
    float th[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = f0 + warp * 4 + i;
      const bool ok = f < n_features;
      pos[i] = ok ? col_offs[f] : 0;
      end[i] = ok ? col_offs[f + 1] : 0;   // the encoder counted exactly these entries
      th[i] = ok ? theta[f] : 0.f;
    }
    // the next 32-word chunk of the bitmap is loaded while this one is scanned
    uint32_t nxt[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int wi = warp + 8 * q, f = f0 + lane;
      nxt[q] = (wi < n_words && f < n_features) ? sbits[static_cast<size_t>(wi) * n_features + f]
                                                : 0u;
    }
    for (int w0 = 0; w0 < n_words; w0 += 32) {
      __syncthreads();
#pragma unroll
      for (int q = 0; q < 4; ++q) tile[warp + 8 * q][lane] = nxt[q];
      __syncthreads();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int wi = w0 + 32 + warp + 8 * q, f = f0 + lane;
        nxt[q] = (wi < n_words && f < n_features)
                     ? sbits[static_cast<size_t>(wi) * n_features + f] : 0u;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int fl = warp * 4 + i;
        const int f = f0 + fl;
        if (f >= n_features) continue;   // uniform per warp
        uint32_t bits = tile[lane][fl];
        const int mine = __popc(bits);
        int incl = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const int tot = __shfl_sync(0xffffffffu, incl, 31);
        int q = pos[i] + incl - mine;
        const int tbase = (w0 + lane) * 32;
        while (bits) {
          const int b = __ffs(bits) - 1;
          bits &= bits - 1;
          if (q < end[i]) csr_tok[q] = tbase + b;
          ++q;
        }
        pos[i] += tot;
      }
    }
    // the entries' pre values and flags: independent loads, 32 in flight per warp
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = f0 + warp * 4 + i;
      if (f >= n_features) continue;
      const uint16_t* prow = pre16 + static_cast<size_t>(f) * ldp;
      const int q1 = min(pos[i], end[i]);
      for (int q = col_offs[f] + lane; q < q1; q += 32) {
        const uint32_t u = prow[csr_tok[q]];
        const float p = __uint_as_float(u << 16);
        csr_val[q] = u | (p > th[i] ? CSR_ACTIVE : 0u) |
                     (fabsf(__fsub_rn(p, th[i])) < eps ? CSR_BAND : 0u);
      }
    }
  }
}

// Sum over the 32 lanes of each of 8 values: after the call, lane l with
// (l & 3) == 0 holds the total of value ((l >> 2) & 7) (a transpose-style
// butterfly: 4 + 2 + 1 exchanges halve the live values, 2 more finish).
__device__ __forceinline__ float warp_sum8(float (&p)[8], int lane) {
  float q4[4], q2[2];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const bool hi = lane & 16;
    const float keep = hi ? p[k + 4] : p[k];
    const float send = hi ? p[k] : p[k + 4];
    q4[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool hi = lane & 8;
    const float keep = hi ? q4[k + 2] : q4[k];
    const float send = hi ? q4[k] : q4[k + 2];
    q2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const bool hi = lane & 4;
  float q = (hi ? q2[1] : q2[0]) + __shfl_xor_sync(0xffffffffu, hi ? q2[0] : q2[1], 4);
  q += __shfl_xor_sync(0xffffffffu, q, 2);
  q += __shfl_xor_sync(0xffffffffu, q, 1);
  return q;
}

// Sum over the 32 lanes of each of 4 values: lane l with (l & 7) == 0 holds
// the total of value ((l >> 3) & 3).
__device__ __forceinline__ float warp_sum4(float (&p)[4], int lane) {
  float q2[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool hi = lane & 16;
    const float keep = hi ? p[k + 2] : p[k];
    const float send = hi ? p[k] : p[k + 2];
    q2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  const bool hi = lane & 8;
  float q = (hi ? q2[1] : q2[0]) + __shfl_xor_sync(0xffffffffu, hi ? q2[0] : q2[1], 8);
  q += __shfl_xor_sync(0xffffffffu, q, 4);
  q += __shfl_xor_sync(0xffffffffu, q, 2);
  q += __shfl_xor_sync(0xffffffffu, q, 1);
  return q;
}

// Two values: lane l with (l & 15) == 0 holds the total of value (l >> 4) & 1.
__device__ __forceinline__ float warp_sum2(float (&p)[2], int lane) {
  const bool hi = lane & 16;
  float q = (hi ? p[1] : p[0]) + __shfl_xor_sync(0xffffffffu, hi ? p[0] : p[1], 16);
  q += __shfl_xor_sync(0xffffffffu, q, 8);
  q += __shfl_xor_sync(0xffffffffu, q, 4);
  q += __shfl_xor_sync(0xffffffffu, q, 2);
  q += __shfl_xor_sync(0xffffffffu, q, 1);
  return q;
}

template <int C>
__device__ __forceinline__ float warp_sum_c(float (&p)[C], int lane) {
  if constexpr (C == 8) return warp_sum8(p, lane);
  else if constexpr (C == 4) return warp_sum4(p, lane);
  else return warp_sum2(p, lane);
}

// Per feature (blocks take features from a global counter; one feature per
// block of d/8 threads, blocks independent): its CSR entries in chunks of C,
//   grad_feat = bf16(go[t] . W_dec[f])   (fp32 accumulation; the bf16 GEMM
//                                          output of 643)
//   active:  dpre = grad_feat; db_enc += dpre; dW_enc[f] += dpre * xc[t];
//            dW_dec[f] += pre * go[t]
//   in band: STE sum += pre * grad_feat + gate_grad
// and at the end the threshold gradient -(sum / 2 eps) * theta. The go and xc
// rows of a chunk are all requested before the first is used. The C dot
// products are reduced by a warp butterfly and one barrier per chunk: every
// thread adds the warps' partials (double-buffered by chunk parity) in the
// same order, so all threads hold the same grad_feat and the result does not
// depend on timing.
template <int C, int U, int MAX_THREADS, int MIN_BLOCKS>
__global__ void __launch_bounds__(MAX_THREADS, MIN_BLOCKS)
    sampled_backward_kernel(const int* __restrict__ col_offs, const int* __restrict__ csr_tok,
                            const uint32_t* __restrict__ csr_val, const bf16* __restrict__ go,
                            const bf16* __restrict__ xc, const bf16* __restrict__ w_dec,
                            const float* __restrict__ theta, int n_features, int n_tokens,
                            int d, float eps, int accumulate, float* __restrict__ g_wdec,
                            float* __restrict__ g_wenc, float* __restrict__ g_logthr,
                            float* __restrict__ g_benc, float* __restrict__ db_enc,
                            int* __restrict__ counter, const SaeB200StepStats* stats,
                            const int* __restrict__ seg_rows = nullptr,
                            int honor_overflow = 1, float* __restrict__ row_sumsq = nullptr) {
  // thread tid owns columns [8 U tid, 8 U tid + 8 U): U consecutive 16-byte vectors.
  // Segment sg of the CSR holds feature seg_rows[sg] (feature sg without seg_rows):
  // the aux-loss backward runs the same kernel over the dead features' entries.
  // row_sumsq != NULL: warp w of the block that finishes feature f writes the sum
  // of squares of its columns of the final (accumulated) W_dec and W_enc gradient
  // rows of f to row_sumsq[f * 32 + w], warp 0 adding the final log_threshold and
  // b_enc gradients of f; warps the block does not have leave their slots alone,
  // so a reader sums the block's warps only. The global gradient norm then needs
  // only these F * warps partials instead of another pass over the gradients.
  if (honor_overflow && stats != nullptr && stats->csr_overflow) return;
  __shared__ int s_f[2];
  __shared__ float s_red[2][32][C];   // [chunk parity][warp][entry]
  const int tid = threadIdx.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  const int nvec = d / 8;
  const bool has = (tid + 1) * U <= nvec;
  const float gate_grad = stats != nullptr ? stats->gate_grad : 0.f;   // (band entries only)
  const uint4* go_v = reinterpret_cast<const uint4*>(go) + U * tid;
  const uint4* xc_v = reinterpret_cast<const uint4*>(xc) + U * tid;
  int it = 0, par = 0;
  if (tid == 0) s_f[0] = atomicAdd(counter, 1);
  __syncthreads();
  while (true) {
    const int sg = s_f[it & 1];
    if (sg >= n_features) break;
    // the next feature is claimed now and published at the end of this one,
    // so the atomic's round trip overlaps this feature's work
    int next = 0;
    if (tid == 0) next = atomicAdd(counter, 1);
    const int s = col_offs[sg], e = col_offs[sg + 1];
    const int f = seg_rows != nullptr ? seg_rows[sg] : sg;
    float wf[8 * U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float w8[8];
      if (has) {
        unpack8(__ldg(reinterpret_cast<const uint4*>(w_dec) + static_cast<size_t>(f) * nvec +
                      U * tid + u), w8);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) w8[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) wf[8 * u + j] = w8[j];
    }
    float ad[8 * U], ae[8 * U];
#pragma unroll
    for (int j = 0; j < 8 * U; ++j) ad[j] = ae[j] = 0.f;
    float thr = 0.f, db = 0.f;
    // entries of the current chunk; those of the next chunk are loaded one
    // chunk ahead, so only the row gathers wait on memory per chunk
    int t[C];
    uint32_t v[C];
#pragma unroll
    for (int r = 0; r < C; ++r) {
      t[r] = s + r < e ? csr_tok[s + r] : 0;
      v[r] = s + r < e ? csr_val[s + r] : 0u;
    }
    for (int i0 = s; i0 < e; i0 += C) {
      const int n = min(C, e - i0);
      int tn[C];
      uint32_t vn[C];
#pragma unroll
      for (int r = 0; r < C; ++r) {
        const int k = i0 + C + r;
        tn[r] = k < e ? csr_tok[k] : 0;
        vn[r] = k < e ? csr_val[k] : 0u;
      }
      // (the clamp only guards the row reads; the fill writes tokens < n_tokens)
#pragma unroll
      for (int r = 0; r < C; ++r) t[r] = min(max(t[r], 0), n_tokens - 1);
      uint4 gu[C][U], xu[C][U];
#pragma unroll
      for (int r = 0; r < C; ++r) {
        const bool ok = has && r < n;
        const bool act = ok && (v[r] & CSR_ACTIVE);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          gu[r][u] = ok ? __ldg(go_v + static_cast<size_t>(t[r]) * nvec + u)
                        : make_uint4(0, 0, 0, 0);
          xu[r][u] = act ? __ldg(xc_v + static_cast<size_t>(t[r]) * nvec + u)
                         : make_uint4(0, 0, 0, 0);
        }
      }
      float part[C];
#pragma unroll
      for (int r = 0; r < C; ++r) {
        // even and odd columns in the two halves of packed FMAs; an active
        // entry's dW_dec term (pre * go, independent of grad_feat) is added
        // while its go values are unpacked
        const bool act = r < n && (v[r] & CSR_ACTIVE);   // uniform across the block
        const float p = __uint_as_float(v[r] << 16);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float g8[8];
          unpack8(gu[r][u], g8);
#pragma unroll
          for (int j = 0; j < 8; j += 2)
            fma2(a0, a1, g8[j], g8[j + 1], wf[8 * u + j], wf[8 * u + j + 1]);
          if (act) {
#pragma unroll
            for (int j = 0; j < 8; j += 2)
              fma2(ad[8 * u + j], ad[8 * u + j + 1], p, p, g8[j], g8[j + 1]);
          }
        }
        part[r] = a0 + a1;
      }
      const float q = warp_sum_c<C>(part, lane);
      constexpr int kStride = 32 / C;
      if ((lane & (kStride - 1)) == 0) s_red[par][wid][lane / kStride] = q;
      __syncthreads();
#pragma unroll
      for (int r = 0; r < C; ++r) {
        if (r < n) {
          float a = 0.f;
          for (int w = 0; w < nw; ++w) a += s_red[par][w][r];
          const float gfv = bf16_round(a);
          const float p = __uint_as_float(v[r] << 16);
          if (v[r] & CSR_ACTIVE) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
              float x8[8];
              unpack8(xu[r][u], x8);
#pragma unroll
              for (int j = 0; j < 8; j += 2)
                fma2(ae[8 * u + j], ae[8 * u + j + 1], gfv, gfv, x8[j], x8[j + 1]);
            }
            db += gfv;
          }
          if (v[r] & CSR_BAND) thr += __fadd_rn(__fmul_rn(p, gfv), gate_grad);
        }
      }
      par ^= 1;
#pragma unroll
      for (int r = 0; r < C; ++r) {
        t[r] = tn[r];
        v[r] = vn[r];
      }
    }
    float sq = 0.f;
    if (has) {
      const size_t o = static_cast<size_t>(f) * d + static_cast<size_t>(tid) * 8 * U;
#pragma unroll
      for (int q4 = 0; q4 < 2 * U; ++q4) {
        if (g_wdec != nullptr) {
          float4* p = reinterpret_cast<float4*>(g_wdec + o) + q4;
          float4 a4 = make_float4(ad[4 * q4], ad[4 * q4 + 1], ad[4 * q4 + 2], ad[4 * q4 + 3]);
          if (accumulate) {
            const float4 u4 = *p;
            a4.x += u4.x; a4.y += u4.y; a4.z += u4.z; a4.w += u4.w;
          }
          *p = a4;
          sq = fmaf(a4.x, a4.x, sq); sq = fmaf(a4.y, a4.y, sq);
          sq = fmaf(a4.z, a4.z, sq); sq = fmaf(a4.w, a4.w, sq);
        }
        float4* p = reinterpret_cast<float4*>(g_wenc + o) + q4;
        float4 e4 = make_float4(ae[4 * q4], ae[4 * q4 + 1], ae[4 * q4 + 2], ae[4 * q4 + 3]);
        if (accumulate) {
          const float4 u4 = *p;
          e4.x += u4.x; e4.y += u4.y; e4.z += u4.z; e4.w += u4.w;
        }
        *p = e4;
        sq = fmaf(e4.x, e4.x, sq); sq = fmaf(e4.y, e4.y, sq);
        sq = fmaf(e4.z, e4.z, sq); sq = fmaf(e4.w, e4.w, sq);
      }
    }
    if (tid == 0) {
      const float gl = -(thr / (eps + eps)) * theta[f];
      const float glv = accumulate ? g_logthr[f] + gl : gl;
      const float gbv = accumulate ? g_benc[f] + db : db;
      g_logthr[f] = glv;
      g_benc[f] = gbv;
      db_enc[f] = db;
      sq = fmaf(glv, glv, sq);
      sq = fmaf(gbv, gbv, sq);
    }
    if (row_sumsq != nullptr) {
      sq = warp_sum(sq);
      if (lane == 0) row_sumsq[static_cast<size_t>(f) * 32 + wid] = sq;
    }
    ++it;
    if (tid == 0) s_f[it & 1] = next;
    __syncthreads();
  }
}



// ------------------------------------------------------------------ decode
// One block per token (grid-stride). The block is G row groups of V threads;
// thread (g, c) owns columns [8c, 8c + 8) and decoder rows g, g + G, ... of the
// token's active list, so a token with thousands of active features is
// gathered G x 8 rows at a time per column slice. The active features are
// extracted from the token's mask row in feature order, their bf16 decoder
// rows gathered with 128-bit loads and accumulated in fp32; the G partial
// sums are combined in a fixed order. Then x_hat = bf16(sum) + b_dec (the
// reference's bf16 GEMM output plus the fp32 bias, 924), r = x - x_hat,
// squared error per token, and the loss gradient go = -(scale * 2r) stored as
// bf16 (what the decoder GEMMs see).
//
// 8 consecutive x values as fp32.
template <typename XT>
__device__ __forceinline__ void load_x8(const XT* x, float (&xv)[8]) {
  if constexpr (sizeof(XT) == 2) {
    unpack8(*reinterpret_cast<const uint4*>(x), xv);
  } else {
    const float4 a = *reinterpret_cast<const float4*>(x);
    const float4 c = *reinterpret_cast<const float4*>(x + 4);
    xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
    xv[4] = c.x; xv[5] = c.y; xv[6] = c.z; xv[7] = c.w;
  }
}

// Residual of 8 columns of one token given the fp32 decoder sum acc and x:
// x_hat = bf16(acc) + b_dec, r = x - x_hat, go = -(scale * 2r) (bf16), and the
// running per-column go sums. Returns the 8 columns' squared error.
__device__ __forceinline__ float residual8_x(const float (&acc)[8], const float (&xv)[8],
                                             const float* __restrict__ b_dec, size_t base, int c0,
                                             float go_scale, bf16* __restrict__ go,
                                             float* __restrict__ x_hat, float (&gsum)[8]) {
  float gv[8], xh[8];
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    xh[j] = __fadd_rn(bf16_round(acc[j]), b_dec[c0 + j]);
    const float r = __fsub_rn(xv[j], xh[j]);
    sq = fmaf(r, r, sq);
    gv[j] = -__fmul_rn(go_scale, __fadd_rn(r, r));
    gsum[j] += gv[j];
  }
  *reinterpret_cast<uint4*>(go + base) = pack8(gv);
  if (x_hat != nullptr) {
    *reinterpret_cast<float4*>(x_hat + base) = make_float4(xh[0], xh[1], xh[2], xh[3]);
    *reinterpret_cast<float4*>(x_hat + base + 4) = make_float4(xh[4], xh[5], xh[6], xh[7]);
  }
  return sq;
}

template <typename XT>
__device__ __forceinline__ float residual8(const float (&acc)[8], const XT* __restrict__ x,
                                           const float* __restrict__ b_dec, size_t base, int c0,
                                           float go_scale, bf16* __restrict__ go,
                                           float* __restrict__ x_hat, float (&gsum)[8]) {
  float xv[8];
  load_x8(x + base, xv);
  return residual8_x(acc, xv, b_dec, base, c0, go_scale, go, x_hat, gsum);
}

// Asynchronous global -> shared copies (LDGSTS): staged without registers.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// x == NULL (inference): the block writes x_hat (fp32, required) and the
// token's active count only.
// partial != NULL (dictionary-sharded step): instead of the residual, the
// block writes the token's fp32 decoder sum over this shard's features to
// partial[b * d + c] and its active count to partial[n_tokens * d + b] (as a
// float); the shards' partials are summed across GPUs and residual_kernel
// finishes the forward.
// The token's x columns are copied into shared memory (cp.async) when its
// decode starts, so that they have landed by the residual; the token after
// next is looked up one token ahead.
// 56 registers: 3 blocks of 384 threads (2 row groups at d = 1536) or 4 of
// 288 (1 row group at d = 2304) per SM; any block of up to 1024 threads fits.
template <typename XT, int G, int RB = 8>
__global__ void __maxnreg__(56)
    decode_kernel(const uint32_t* __restrict__ mask, const bf16* __restrict__ pre,
                  const bf16* __restrict__ w_dec, const float* __restrict__ b_dec,
                  const XT* __restrict__ x, int64_t n_tokens, int d, int n_features,
                  int mask_words, int ldp, float go_scale, bf16* __restrict__ go,
                  float* __restrict__ x_hat, float* __restrict__ tok_sqerr,
                  int* __restrict__ tok_cnt, float* __restrict__ gosum_part,
                  float* __restrict__ partial, const int* __restrict__ order) {
  __shared__ int s_f[DECODE_LIST_CAP];
  __shared__ uint32_t s_pw[DECODE_LIST_CAP];   // the words holding the entries' pre values
  __shared__ int s_itmp[33];
  __shared__ float s_ftmp[33];
  // dynamic: (G - 1) x V x 2 float4 partial sums, then for the residual
  // (x != NULL, partial == NULL): V x 2 float4 go sums | V x 8 XT x values
  extern __shared__ float4 s_dyn[];
  const int tid = threadIdx.x;
  const int V = blockDim.x / G;
  const int g = tid / V;
  const int col = tid - g * V;
  const int nvec = d / 8;
  const bool has = col < nvec;
  const int wpt = (mask_words + blockDim.x - 1) / blockDim.x;
  const int w0 = min(mask_words, tid * wpt);
  const int w1 = min(mask_words, w0 + wpt);
  float4* s_part = s_dyn;
  float4* s_gsum = s_dyn + (G - 1) * V * 2;   // this block's per-column go sums
  XT* s_x = reinterpret_cast<XT*>(s_gsum + V * 2);
  const bool residual = partial == nullptr && x != nullptr;   // uniform
  const bool stage_x = residual && g == 0 && has;

  if (stage_x) {
    s_gsum[col * 2] = make_float4(0.f, 0.f, 0.f, 0.f);
    s_gsum[col * 2 + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  auto token_at = [&](int64_t k) -> int {
    return k < n_tokens ? (order != nullptr ? order[k] : static_cast<int>(k)) : -1;
  };
  int b = token_at(blockIdx.x);
  int bn = token_at(blockIdx.x + static_cast<int64_t>(gridDim.x));
  for (int64_t k = blockIdx.x; k < n_tokens; k += gridDim.x) {
    const int bnn = token_at(k + 2 * static_cast<int64_t>(gridDim.x));
    if (stage_x) {
      const XT* xs = x + static_cast<size_t>(b) * d + col * 8;
      cp_async16(s_x + col * 8, xs);
      if constexpr (sizeof(XT) == 4) cp_async16(s_x + col * 8 + 4, xs + 4);
      cp_async_commit();
    }
    const uint32_t* mrow = mask + static_cast<size_t>(b) * mask_words;
    int mine = 0;
    for (int w = w0; w < w1; ++w) mine += __popc(mrow[w]);
    int total = 0;
    const int my_off = block_excl_scan(mine, s_itmp, total);

    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;

    const uint32_t* pre_w = reinterpret_cast<const uint32_t*>(pre);
    const bool hi_half = b & 1;   // ldp is even: the token's parity picks the half of a word
    for (int win = 0; win < total; win += DECODE_LIST_CAP) {
      __syncthreads();
      // the active features in feature order; the 4-byte words holding their
      // pre values are copied by cp.async, so that their round trip overlaps
      // the first row batch's instead of preceding it
      if (my_off < win + DECODE_LIST_CAP && my_off + mine > win) {
        int rank = my_off;
        for (int w = w0; w < w1; ++w) {
          uint32_t bits = mrow[w];
          while (bits) {
            const int bit = __ffs(bits) - 1;
            bits &= bits - 1;
            if (rank >= win && rank < win + DECODE_LIST_CAP) {
              const int f = w * 32 + bit;
              s_f[rank - win] = f;
              cp_async4(&s_pw[rank - win], pre_w + ((static_cast<size_t>(f) * ldp + b) >> 1));
            }
            ++rank;
          }
        }
      }
      cp_async_commit();
      __syncthreads();   // the feature ids are in place
      const int n = min(DECODE_LIST_CAP, total - win);
      const uint4* wcol = reinterpret_cast<const uint4*>(w_dec) + col;
      auto pre_at = [&](int k) {
        const uint32_t wd = s_pw[k];
        return hi_half ? bf_hi(wd) : bf_lo(wd);
      };
      // rows g, g + G, g + 2G, ... of the list in order, RB loads in flight
      int i = g;
      uint4 u[RB];
      // the first batch's loads go out before the wait for the pre words
#pragma unroll
      for (int r = 0; r < RB; ++r)
        u[r] = (has && i < n) ? __ldg(wcol + static_cast<size_t>(s_f[min(i + r * G, n - 1)]) * nvec)
                              : make_uint4(0u, 0u, 0u, 0u);
      cp_async_wait<0>();
      __syncthreads();   // every thread's pre words (and x columns) have landed
      if (has) {
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (i + r * G < n) {
            float wf[8];
            unpack8(u[r], wf);
            const float a = pre_at(i + r * G);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(a, wf[j], acc[j]);
          }
        }
        i += RB * G;
        for (; i + (RB - 1) * G < n; i += RB * G) {
#pragma unroll
          for (int r = 0; r < RB; ++r)
            u[r] = __ldg(wcol + static_cast<size_t>(s_f[i + r * G]) * nvec);
#pragma unroll
          for (int r = 0; r < RB; ++r) {
            float wf[8];
            unpack8(u[r], wf);
            const float a = pre_at(i + r * G);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(a, wf[j], acc[j]);
          }
        }
        for (; i < n; i += G) {
          float wf[8];
          unpack8(__ldg(wcol + static_cast<size_t>(s_f[i]) * nvec), wf);
          const float a = pre_at(i);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = fmaf(a, wf[j], acc[j]);
        }
      }
    }
    if constexpr (G > 1) {
      __syncthreads();
      if (g > 0 && has) {
        s_part[((g - 1) * V + col) * 2] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        s_part[((g - 1) * V + col) * 2 + 1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      }
      __syncthreads();
      if (g == 0 && has) {
#pragma unroll
        for (int h = 0; h < G - 1; ++h) {
          const float4 a = s_part[(h * V + col) * 2];
          const float4 c = s_part[(h * V + col) * 2 + 1];
          acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
          acc[4] += c.x; acc[5] += c.y; acc[6] += c.z; acc[7] += c.w;
        }
      }
    }

    const int bt = b;
    b = bn;
    bn = bnn;
    const size_t base = static_cast<size_t>(bt) * d + col * 8;
    if (partial != nullptr) {   // uniform across the block
      if (g == 0 && has) {
        *reinterpret_cast<float4*>(partial + base) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(partial + base + 4) =
            make_float4(acc[4], acc[5], acc[6], acc[7]);
      }
      if (tid == 0) partial[n_tokens * d + bt] = static_cast<float>(total);
      continue;
    }
    if (x == nullptr) {         // inference: x_hat only (uniform across the block)
      if (g == 0 && has) {
        float xh[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) xh[j] = __fadd_rn(bf16_round(acc[j]), b_dec[col * 8 + j]);
        *reinterpret_cast<float4*>(x_hat + base) = make_float4(xh[0], xh[1], xh[2], xh[3]);
        *reinterpret_cast<float4*>(x_hat + base + 4) = make_float4(xh[4], xh[5], xh[6], xh[7]);
      }
      if (tid == 0) tok_cnt[bt] = total;
      continue;
    }
    float sq = 0.f;
    if (stage_x) {
      cp_async_wait<0>();   // this thread's x columns have landed
      float xv[8], gsum[8];
      load_x8(s_x + col * 8, xv);
      const float4 g0 = s_gsum[col * 2], g1 = s_gsum[col * 2 + 1];
      gsum[0] = g0.x; gsum[1] = g0.y; gsum[2] = g0.z; gsum[3] = g0.w;
      gsum[4] = g1.x; gsum[5] = g1.y; gsum[6] = g1.z; gsum[7] = g1.w;
      sq = residual8_x(acc, xv, b_dec, base, col * 8, go_scale, go, x_hat, gsum);
      s_gsum[col * 2] = make_float4(gsum[0], gsum[1], gsum[2], gsum[3]);
      s_gsum[col * 2 + 1] = make_float4(gsum[4], gsum[5], gsum[6], gsum[7]);
    }
    const float tot_sq = block_sum(sq, s_ftmp);
    if (tid == 0) {
      tok_sqerr[bt] = tot_sq;
      tok_cnt[bt] = total;
    }
  }
  if (stage_x) {
    float4* dst = reinterpret_cast<float4*>(gosum_part + static_cast<size_t>(blockIdx.x) * d + col * 8);
    dst[0] = s_gsum[col * 2];
    dst[1] = s_gsum[col * 2 + 1];
  }
  // sharded step: the partials may be read by other GPUs (peer exchange)
  if (partial != nullptr) __threadfence_system();
}

// Per token: its active count (popcount of the mask row) and its id, the
// keys and values of the decode-order sort. One warp per token.
__global__ void __launch_bounds__(256)
    token_count_kernel(const uint32_t* __restrict__ mask, int64_t n_tokens, int mask_words,
                       int* __restrict__ counts, int* __restrict__ ids) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t b = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
       b < n_tokens; b += warps) {
    const uint32_t* row = mask + b * mask_words;
    int c = 0;
    for (int w = lane; w < mask_words; w += 32) c += __popc(row[w]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) {
      counts[b] = c;
      ids[b] = static_cast<int>(b);
    }
  }
}

// Second half of the dictionary-sharded forward: xsum holds the decoder sums
// and active counts of decode_kernel's partial mode, already summed over all
// shards ([n_tokens * d] floats, then [n_tokens] counts). Same residual, loss
// and go as decode_kernel, one block of d / 8 threads per token (grid-stride,
// launched with DECODE_GRID blocks so that gosum_part has the same rows).
template <typename XT>
__global__ void __launch_bounds__(1024)
    residual_kernel(const float* __restrict__ xsum, const float* __restrict__ b_dec,
                    const XT* __restrict__ x, int64_t n_tokens, int d, float go_scale,
                    bf16* __restrict__ go, float* __restrict__ x_hat,
                    float* __restrict__ tok_sqerr, int* __restrict__ tok_cnt,
                    float* __restrict__ gosum_part) {
  __shared__ float s_ftmp[33];
  const int col = threadIdx.x;
  const bool has = col < d / 8;
  float gsum[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) gsum[j] = 0.f;
  for (int64_t b = blockIdx.x; b < n_tokens; b += gridDim.x) {
    float sq = 0.f;
    if (has) {
      const size_t base = static_cast<size_t>(b) * d + col * 8;
      const float4 a = *reinterpret_cast<const float4*>(xsum + base);
      const float4 c = *reinterpret_cast<const float4*>(xsum + base + 4);
      const float acc[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
      sq = residual8(acc, x, b_dec, base, col * 8, go_scale, go, x_hat, gsum);
    }
    const float tot_sq = block_sum(sq, s_ftmp);
    if (threadIdx.x == 0) {
      tok_sqerr[b] = tot_sq;
      tok_cnt[b] = static_cast<int>(xsum[n_tokens * d + b]);
    }
  }
  if (has) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      gosum_part[static_cast<size_t>(blockIdx.x) * d + col * 8 + j] = gsum[j];
  }
}

// Loss terms of the microbatch and the sparsity gradient reaching each gate
// element (2963-2974): slack = max(0, l0 - target),
// d sparsity / d gate = (lambda + mu * slack) / accum / B where l0 >= target
// (torch.clamp passes the gradient at the boundary).
__global__ void __launch_bounds__(1024)
    forward_stats_kernel(const float* __restrict__ tok_sqerr, const int* __restrict__ tok_cnt,
                         int64_t n_tokens, int d, float lambda_l0, float al_mu, float target,
                         int accum, SaeB200StepStats* stats) {
  __shared__ float s_tmp[33];
  __shared__ unsigned long long s_cnt;
  if (threadIdx.x == 0) s_cnt = 0;
  // 8 loads in flight per thread; partial sums in a fixed order
  float sq = 0.f;
  unsigned long long cnt = 0;
  const int64_t step = static_cast<int64_t>(blockDim.x) * 8;
  int64_t i0 = threadIdx.x;
  for (; i0 + 7 * blockDim.x < n_tokens; i0 += step) {
    float a[8];
    int c[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      a[u] = tok_sqerr[i0 + u * blockDim.x];
      c[u] = tok_cnt[i0 + u * blockDim.x];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      sq += a[u];
      cnt += static_cast<unsigned long long>(c[u]);
    }
  }
  for (int64_t i = i0; i < n_tokens; i += blockDim.x) {
    sq += tok_sqerr[i];
    cnt += static_cast<unsigned long long>(tok_cnt[i]);
  }
  const float total_sq = block_sum(sq, s_tmp);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(&s_cnt, cnt);   // integer: exact in any order
  __syncthreads();
  if (threadIdx.x == 0) {
    const float inv_accum = 1.0f / static_cast<float>(accum);
    const float recon = (total_sq / static_cast<float>(static_cast<double>(n_tokens) * d)) * inv_accum;
    const float l0 = static_cast<float>(s_cnt) / static_cast<float>(n_tokens);
    const float diff = l0 - target;
    const float slack = fmaxf(diff, 0.f);
    const float sparsity = (lambda_l0 * slack + 0.5f * al_mu * slack * slack) * inv_accum;
    const float ggrad =
        diff >= 0.f ? ((lambda_l0 + al_mu * slack) * inv_accum) / static_cast<float>(n_tokens) : 0.f;
    stats->recon_loss = recon;
    stats->aux_loss = 0.f;   // sae_b200_aux_forward sets it when the aux loss is on
    stats->l0 = l0;
    stats->sparsity_loss = sparsity;
    stats->gate_grad = ggrad;
    stats->loss = recon + sparsity;
  }
}

// ------------------------------------------------------- backward reductions
// Per feature: the threshold STE gradient -(sum / (2 eps)) * theta and the
// encoder-bias gradient (column sum of the gated grad_feat, 597-600).
__global__ void feature_grads_kernel(const float* __restrict__ thr_part,
                                     const float* __restrict__ dbenc_part,
                                     const float* __restrict__ theta, int n_tiles, int n_features,
                                     float eps, int accumulate, float* __restrict__ g_logthr,
                                     float* __restrict__ g_benc, float* __restrict__ db_enc) {
  for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < n_features;
       f += gridDim.x * blockDim.x) {
    float thr = 0.f, db = 0.f;
    for (int t = 0; t < n_tiles; ++t) {
      const size_t i = static_cast<size_t>(t) * n_features + f;
      thr += thr_part[i];
      db += dbenc_part[i];
    }
    const float g = -(thr / (eps + eps)) * theta[f];
    g_logthr[f] = accumulate ? g_logthr[f] + g : g;
    g_benc[f] = accumulate ? g_benc[f] + db : db;
    db_enc[f] = db;
  }
}

// Partial GEMV for the reassociated b_dec gradient -(sum_b dpre) W_enc (601).
__global__ void __launch_bounds__(1024)
    bdec_gemv_kernel(const float* __restrict__ db_enc, const bf16* __restrict__ w_enc,
                     int n_features, int d, float* __restrict__ part) {
  const int nvec = d / 8;
  const int tid = threadIdx.x;
  if (tid >= nvec) return;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  const uint4* wv = reinterpret_cast<const uint4*>(w_enc) + tid;
  // 8 rows in flight per thread, requested together with their coefficients
  // (not after them: almost every feature fires in a microbatch); a zero
  // coefficient (feature without active tokens) skips its FMAs, keeping the
  // fixed summation order
  int f = blockIdx.x;
  for (; f + 7 * static_cast<int>(gridDim.x) < n_features; f += 8 * gridDim.x) {
    float sc[8];
    uint4 u[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int fr = f + r * gridDim.x;
      sc[r] = db_enc[fr];
      u[r] = __ldg(wv + static_cast<size_t>(fr) * nvec);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (sc[r] == 0.f) continue;
      float wf[8];
      unpack8(u[r], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = fmaf(sc[r], wf[j], acc[j]);
    }
  }
  for (; f < n_features; f += gridDim.x) {
    const float sc = db_enc[f];
    if (sc == 0.f) continue;
    float wf[8];
    unpack8(__ldg(wv + static_cast<size_t>(f) * nvec), wf);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = fmaf(sc, wf[j], acc[j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) part[static_cast<size_t>(blockIdx.x) * d + tid * 8 + j] = acc[j];
}

// b_dec gradient: sum_b go (the fp32 gradient through "+ b_dec", 924) minus
// the reassociated encoder term.
// Block = 32 columns x 32 row lanes; each lane sums every 32nd partial row,
// then the 32 lane sums are added in a fixed order.
__global__ void __launch_bounds__(1024)
    bdec_grad_kernel(const float* __restrict__ gosum_part, int n_go,
                     const float* __restrict__ gemv_part, int n_gemv, int d, int accumulate,
                     float* __restrict__ g_bdec,
                     const SaeB200StepStats* skip_on_overflow = nullptr) {
  // (the sampled backward, queued before the host has seen the forward's
  // statistics, leaves every gradient untouched when the CSR overflowed)
  if (skip_on_overflow != nullptr && skip_on_overflow->csr_overflow) return;
  __shared__ float s1[32][33];
  __shared__ float s2[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int k = blockIdx.x * 32 + tx;
  float a = 0.f, b = 0.f;
  if (k < d) {
    // (unrolled so that several of the independent loads are in flight; the
    // sums keep their order)
#pragma unroll 8
    for (int i = ty; i < n_go; i += 32) a += gosum_part[static_cast<size_t>(i) * d + k];
#pragma unroll 8
    for (int i = ty; i < n_gemv; i += 32) b += gemv_part[static_cast<size_t>(i) * d + k];
  }
  s1[ty][tx] = a;
  s2[ty][tx] = b;
  __syncthreads();
  if (ty == 0 && k < d) {
    float x = 0.f, y = 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      x += s1[r][tx];
      y += s2[r][tx];
    }
    const float g = x - y;
    g_bdec[k] = accumulate ? g_bdec[k] + g : g;
  }
}

// Sparse decoder / encoder weight gradients over the feature-major CSR:
//   dW_dec[f] = sum_{(t,f) active} pre[t,f] * go[t]     (index_add_, 645-652)
//   dW_enc[f] = sum_{(t,f) active} dpre[t,f] * xc[t]    (dpre^T xc, 599)
// Blocks take features from a global counter. A block is G row groups of V
// threads: thread (g, c) owns columns [8c, 8c + 8) and entries g, g + G, ... of
// the feature's CSR row; the G partial sums are added in a fixed order, so
// the result does not depend on timing.
__device__ __forceinline__ void scatter_fma(uint32_t v, const uint4 gu, const uint4 xu,
                                            float (&ad)[8], float (&ae)[8]) {
  const float a = __uint_as_float(v << 16), q = __uint_as_float(v & 0xFFFF0000u);
  float gf[8], xf[8];
  unpack8(gu, gf);
  unpack8(xu, xf);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    ad[j] = fmaf(a, gf[j], ad[j]);
    ae[j] = fmaf(q, xf[j], ae[j]);
  }
}

template <int G>
__global__ void __launch_bounds__(1024)
    scatter_weight_grads_kernel(const int* __restrict__ col_offs, const int* __restrict__ csr_tok,
                                const uint32_t* __restrict__ csr_val, const bf16* __restrict__ go,
                                const bf16* __restrict__ xc, int n_features, int d,
                                int accumulate, float* __restrict__ g_wdec,
                                float* __restrict__ g_wenc, int* __restrict__ counter,
                                const SaeB200StepStats* stats) {
  if (stats->csr_overflow) return;
  __shared__ int s_f[2];
  extern __shared__ float4 s_part[];   // (G - 1) x V x 4 float4
  const int tid = threadIdx.x;
  const int V = blockDim.x / G;
  const int g = tid / V;
  const int col = tid - g * V;
  const int nvec = d / 8;
  const bool has = col < nvec;
  const uint4* go_v = reinterpret_cast<const uint4*>(go) + col;
  const uint4* xc_v = reinterpret_cast<const uint4*>(xc) + col;
  int it = 0;
  while (true) {
    if (tid == 0) s_f[it & 1] = atomicAdd(counter, 1);
    __syncthreads();
    const int f = s_f[it & 1];
    ++it;
    if (f >= n_features) break;
    const int s = col_offs[f], e = col_offs[f + 1];
    float ad[8], ae[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) ad[j] = ae[j] = 0.f;
    if (has) {
      int i = s + g;
      for (; i + 3 * G < e; i += 4 * G) {
        int t[4];
        uint32_t v[4];
        uint4 gu[4], xu[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          t[r] = csr_tok[i + r * G];
          v[r] = csr_val[i + r * G];
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          gu[r] = __ldg(go_v + static_cast<size_t>(t[r]) * nvec);
          xu[r] = __ldg(xc_v + static_cast<size_t>(t[r]) * nvec);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) scatter_fma(v[r], gu[r], xu[r], ad, ae);
      }
      for (; i < e; i += G) {
        const int t0 = csr_tok[i];
        scatter_fma(csr_val[i], __ldg(go_v + static_cast<size_t>(t0) * nvec),
                    __ldg(xc_v + static_cast<size_t>(t0) * nvec), ad, ae);
      }
    }
    if constexpr (G > 1) {
      if (e - s > 1) {   // uniform across the block
        if (g > 0 && has) {
          float4* p = s_part + ((g - 1) * V + col) * 4;
          p[0] = make_float4(ad[0], ad[1], ad[2], ad[3]);
          p[1] = make_float4(ad[4], ad[5], ad[6], ad[7]);
          p[2] = make_float4(ae[0], ae[1], ae[2], ae[3]);
          p[3] = make_float4(ae[4], ae[5], ae[6], ae[7]);
        }
        __syncthreads();
        if (g == 0 && has) {
#pragma unroll
          for (int h = 0; h < G - 1; ++h) {
            const float4* p = s_part + (h * V + col) * 4;
            const float4 a0 = p[0], a1 = p[1], b0 = p[2], b1 = p[3];
            ad[0] += a0.x; ad[1] += a0.y; ad[2] += a0.z; ad[3] += a0.w;
            ad[4] += a1.x; ad[5] += a1.y; ad[6] += a1.z; ad[7] += a1.w;
            ae[0] += b0.x; ae[1] += b0.y; ae[2] += b0.z; ae[3] += b0.w;
            ae[4] += b1.x; ae[5] += b1.y; ae[6] += b1.z; ae[7] += b1.w;
          }
        }
        __syncthreads();
      }
    }
    if (g == 0 && has) {
      const size_t o = static_cast<size_t>(f) * d + col * 8;
      if (g_wdec != nullptr) {
        float4* p = reinterpret_cast<float4*>(g_wdec + o);
        if (accumulate) {
          const float4 u = p[0], w = p[1];
          ad[0] += u.x; ad[1] += u.y; ad[2] += u.z; ad[3] += u.w;
          ad[4] += w.x; ad[5] += w.y; ad[6] += w.z; ad[7] += w.w;
        }
        p[0] = make_float4(ad[0], ad[1], ad[2], ad[3]);
        p[1] = make_float4(ad[4], ad[5], ad[6], ad[7]);
      }
      float4* p = reinterpret_cast<float4*>(g_wenc + o);
      if (accumulate) {
        const float4 u = p[0], w = p[1];
        ae[0] += u.x; ae[1] += u.y; ae[2] += u.z; ae[3] += u.w;
        ae[4] += w.x; ae[5] += w.y; ae[6] += w.z; ae[7] += w.w;
      }
      p[0] = make_float4(ae[0], ae[1], ae[2], ae[3]);
      p[1] = make_float4(ae[4], ae[5], ae[6], ae[7]);
    }
  }
}

// ------------------------------------------------------------ grad norm
struct GradList {
  const float* p[5];
  int64_t n[5];
};

__global__ void __launch_bounds__(512)
    grad_sumsq_kernel(GradList gl, float* __restrict__ part) {
  __shared__ float s_tmp[33];
  float acc = 0.f;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int k = 0; k < 5; ++k) {
    const float* p = gl.p[k];
    if (p == nullptr) continue;
    const int64_t n = gl.n[k];
    const int64_t n4 = n / 4;
    const float4* p4 = reinterpret_cast<const float4*>(p);
    for (int64_t i = tid; i < n4; i += stride) {
      const float4 v = p4[i];
      acc = fmaf(v.x, v.x, acc);
      acc = fmaf(v.y, v.y, acc);
      acc = fmaf(v.z, v.z, acc);
      acc = fmaf(v.w, v.w, acc);
    }
    for (int64_t i = n4 * 4 + tid; i < n; i += stride) acc = fmaf(p[i], p[i], acc);
  }
  const float s = block_sum(acc, s_tmp);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

// Sum of squares for the global gradient norm after the sampled backward:
// part[block] = sum of the row_sumsq partials (32 slots per feature, the first
// n_warps of each filled) + the squares of the gradients in gl (those the
// sampled backward does not cover: the b_dec gradient, and a W_dec gradient
// buffer when the decoder is frozen). Fixed order: deterministic.
__global__ void __launch_bounds__(512)
    grad_sumsq_rows_kernel(const float* __restrict__ row_sumsq, int64_t n_features, int n_warps,
                           GradList gl, float* __restrict__ part) {
  __shared__ float s_tmp[33];
  float acc = 0.f;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t n_slots = n_features * n_warps;
  for (int64_t i = tid; i < n_slots; i += stride)
    acc += row_sumsq[(i / n_warps) * 32 + i % n_warps];
  for (int k = 0; k < 5; ++k) {
    const float* p = gl.p[k];
    if (p == nullptr) continue;
    for (int64_t i = tid; i < gl.n[k]; i += stride) acc = fmaf(p[i], p[i], acc);
  }
  const float s = block_sum(acc, s_tmp);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

__global__ void grad_norm_final_kernel(const float* __restrict__ part, int n_part, float max_norm,
                                       SaeB200StepStats* stats) {
  __shared__ float s_tmp[33];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n_part; i += blockDim.x) acc += part[i];
  const float s = block_sum(acc, s_tmp);
  if (threadIdx.x == 0) {
    const float norm = sqrtf(s);
    const float coef = max_norm / (norm + 1e-6f);
    stats->grad_norm = norm;
    stats->clip_coef = fminf(coef, 1.0f);
  }
}

// out[0] = sum of the n_part per-block sums of squares (fixed order); the
// dictionary-sharded step adds this partial over the shards before the norm.
__global__ void sum_parts_kernel(const float* __restrict__ part, int n_part,
                                 float* __restrict__ out) {
  __shared__ float s_tmp[33];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n_part; i += blockDim.x) acc += part[i];
  const float s = block_sum(acc, s_tmp);
  if (threadIdx.x == 0) out[0] = s;
}

// -------------------------------------------------------------------- Adam
struct AdamScalars {
  float lr, beta1, beta2, eps, wd, grad_scale, step_size, bc2_sqrt;
  int use_clip;
};

__device__ __forceinline__ float adam_update(float p, float g, float& m, float& v,
                                             const AdamScalars& h, float clip) {
  if (h.use_clip) g = g * clip;
  if (h.grad_scale != 1.0f) g = g * h.grad_scale;
  if (h.wd != 0.f) g = g + p * h.wd;
  m = h.beta1 * m + (1.f - h.beta1) * g;
  v = h.beta2 * v + (1.f - h.beta2) * g * g;
  const float denom = sqrtf(v) / h.bc2_sqrt + h.eps;
  return p - h.step_size * m / denom;
}

// One warp per row of a [rows, cols] weight (cols % 4 == 0, cols <= 128*MAXV):
// Adam on the row, optional renormalisation of the updated row to unit L2
// norm (clamped at 1e-8), fp32 write-back and bf16 copy.
template <int MAXV>
__global__ void __launch_bounds__(256)
    adam_rows_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                     float* __restrict__ v, bf16* __restrict__ shadow, int64_t rows, int cols,
                     AdamScalars h, const SaeB200StepStats* stats, int renorm) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int nv = cols / 4;
  const float clip = (h.use_clip && stats != nullptr) ? stats->clip_coef : 1.f;
  for (int64_t r = warp; r < rows; r += nwarps) {
    float4* p4 = reinterpret_cast<float4*>(p + r * cols);
    const float4* g4 = reinterpret_cast<const float4*>(g + r * cols);
    float4* m4 = reinterpret_cast<float4*>(m + r * cols);
    float4* v4 = reinterpret_cast<float4*>(v + r * cols);
    float4 pr[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int idx = lane + 32 * i;
      if (idx < nv) {
        float4 pp = p4[idx];
        const float4 gg = g4[idx];
        float4 mm = m4[idx], vv = v4[idx];
        pp.x = adam_update(pp.x, gg.x, mm.x, vv.x, h, clip);
        pp.y = adam_update(pp.y, gg.y, mm.y, vv.y, h, clip);
        pp.z = adam_update(pp.z, gg.z, mm.z, vv.z, h, clip);
        pp.w = adam_update(pp.w, gg.w, mm.w, vv.w, h, clip);
        m4[idx] = mm;
        v4[idx] = vv;
        pr[i] = pp;
        ss += pp.x * pp.x + pp.y * pp.y + pp.z * pp.z + pp.w * pp.w;
      }
    }
    float nrm = 1.f;
    if (renorm) nrm = fmaxf(sqrtf(warp_sum(ss)), 1e-8f);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int idx = lane + 32 * i;
      if (idx < nv) {
        float4 pp = pr[i];
        if (renorm) {
          pp.x = __fdiv_rn(pp.x, nrm);
          pp.y = __fdiv_rn(pp.y, nrm);
          pp.z = __fdiv_rn(pp.z, nrm);
          pp.w = __fdiv_rn(pp.w, nrm);
        }
        p4[idx] = pp;
        if (shadow != nullptr) {
          uint2 u;
          u.x = pack2(pp.x, pp.y);
          u.y = pack2(pp.z, pp.w);
          reinterpret_cast<uint2*>(shadow + r * cols)[idx] = u;
        }
      }
    }
  }
}

// Wide rows: TPR = cols / (4 VPT) threads (a multiple of 32) share a row, each
// holding VPT float4 of it in registers; a block holds RPB rows, and the row
// norm is a warp sum plus a fixed-order sum over the row's warps. All loads of
// a thread are issued before the first use, so a warp keeps 4 VPT 16-byte
// loads in flight -- the wide-row replacement of the warp-per-row kernel, whose
// per-lane register array grows with the row width.
template <int VPT>
__global__ void __launch_bounds__(512)
    adam_rows_wide_kernel(float* __restrict__ p, const float* __restrict__ g,
                          float* __restrict__ m, float* __restrict__ v, bf16* __restrict__ shadow,
                          int64_t rows, int cols, int tpr, AdamScalars h,
                          const SaeB200StepStats* stats, int renorm) {
  __shared__ float s_ss[32];
  const int rpb = blockDim.x / tpr;
  const int rl = threadIdx.x / tpr;            // row slot in the block
  const int c = threadIdx.x - rl * tpr;        // thread within the row
  const int wir = c >> 5, lane = threadIdx.x & 31;
  const int wpr = tpr >> 5;                    // warps per row
  const float clip = (h.use_clip && stats != nullptr) ? stats->clip_coef : 1.f;
  for (int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpb; r0 < rows;
       r0 += static_cast<int64_t>(gridDim.x) * rpb) {
    const int64_t r = r0 + rl;
    const bool ok = rl < rpb && r < rows;
    float4 pr[VPT], gr[VPT], mr[VPT], vr[VPT];
    const size_t base = static_cast<size_t>(ok ? r : 0) * cols;
    float4* p4 = reinterpret_cast<float4*>(p + base);
    float4* m4 = reinterpret_cast<float4*>(m + base);
    float4* v4 = reinterpret_cast<float4*>(v + base);
    const float4* g4 = reinterpret_cast<const float4*>(g + base);
    if (ok) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = c + tpr * i;
        pr[i] = p4[idx];
        gr[i] = g4[idx];
        mr[i] = m4[idx];
        vr[i] = v4[idx];
      }
    }
    float ss = 0.f;
    if (ok) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = c + tpr * i;
        float4 pp = pr[i], mm = mr[i], vv = vr[i];
        const float4 gg = gr[i];
        pp.x = adam_update(pp.x, gg.x, mm.x, vv.x, h, clip);
        pp.y = adam_update(pp.y, gg.y, mm.y, vv.y, h, clip);
        pp.z = adam_update(pp.z, gg.z, mm.z, vv.z, h, clip);
        pp.w = adam_update(pp.w, gg.w, mm.w, vv.w, h, clip);
        m4[idx] = mm;
        v4[idx] = vv;
        pr[i] = pp;
        ss += pp.x * pp.x + pp.y * pp.y + pp.z * pp.z + pp.w * pp.w;
      }
    }
    float nrm = 1.f;
    if (renorm) {
      ss = warp_sum(ss);
      __syncthreads();
      if (lane == 0 && rl < rpb) s_ss[rl * wpr + wir] = ss;
      __syncthreads();
      if (ok) {
        float t = 0.f;
        for (int w = 0; w < wpr; ++w) t += s_ss[rl * wpr + w];
        nrm = fmaxf(sqrtf(t), 1e-8f);
      }
    }
    if (ok) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int idx = c + tpr * i;
        float4 pp = pr[i];
        if (renorm) {
          pp.x = __fdiv_rn(pp.x, nrm);
          pp.y = __fdiv_rn(pp.y, nrm);
          pp.z = __fdiv_rn(pp.z, nrm);
          pp.w = __fdiv_rn(pp.w, nrm);
        }
        p4[idx] = pp;
        if (shadow != nullptr) {
          uint2 u;
          u.x = pack2(pp.x, pp.y);
          u.y = pack2(pp.z, pp.w);
          reinterpret_cast<uint2*>(shadow + base)[idx] = u;
        }
      }
    }
  }
}

// Elementwise Adam for the vectors (b_enc, b_dec, log_threshold) and for
// weights too wide for the row kernel.
__global__ void adam_flat_kernel(float* __restrict__ p, const float* __restrict__ g,
                                 float* __restrict__ m, float* __restrict__ v, int64_t n,
                                 AdamScalars h, const SaeB200StepStats* stats) {
  const float clip = (h.use_clip && stats != nullptr) ? stats->clip_coef : 1.f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float mm = m[i], vv = v[i];
    p[i] = adam_update(p[i], g[i], mm, vv, h, clip);
    m[i] = mm;
    v[i] = vv;
  }
}

}  // namespace sae
