// CUDA-core kernels behind the dense pieces of the module API (encode_pre in
// fp32, jumprelu forward/backward on dense tensors, dense decode and its
// gradients) and the dense backward used when a microbatch's active set
// does not fit the sparse workspace.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include "step_kernels.cuh"

namespace sae {

template <typename T>
__device__ __forceinline__ float load_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_f<float>(const float* p, int64_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float load_f<bf16>(const bf16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ void store_f(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void store_f<float>(float* p, int64_t i, float v) {
  p[i] = v;
}
template <>
__device__ __forceinline__ void store_f<bf16>(bf16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

// C[m, n] = alpha * sum_k A[m, k] B[n, k] + beta * C[m, n] + bias[n]
// 64 x 64 output tile per block, 256 threads x (4 x 4) outputs, K slabs of 16.
constexpr int GG_T = 64;
constexpr int GG_K = 16;

template <typename TA, typename TB, typename TC>
__global__ void __launch_bounds__(256)
    gemm_generic_kernel(int64_t M, int64_t N, int64_t K, float alpha, const TA* __restrict__ A,
                        int64_t sam, int64_t sak, const TB* __restrict__ B, int64_t sbn,
                        int64_t sbk, float beta, TC* __restrict__ C, int64_t scm, int64_t scn,
                        const float* __restrict__ bias) {
  __shared__ float s_a[GG_K][GG_T + 1];
  __shared__ float s_b[GG_K][GG_T + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * GG_T;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * GG_T;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += GG_K) {
    for (int i = threadIdx.x; i < GG_T * GG_K; i += 256) {
      const int r = i % GG_T, kk = i / GG_T;
      const int64_t gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      s_a[kk][r] = (gm < M && gk < K) ? load_f(A, gm * sam + gk * sak) : 0.f;
      s_b[kk][r] = (gn < N && gk < K) ? load_f(B, gn * sbn + gk * sbk) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < GG_K; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = s_a[kk][ty + 16 * i];
        b[i] = s_b[kk][tx + 16 * i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty + 16 * i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx + 16 * j;
      if (gn >= N) continue;
      const int64_t ci = gm * scm + gn * scn;
      float v = alpha * acc[i][j];
      if (beta != 0.f) v = fmaf(beta, load_f(C, ci), v);
      if (bias != nullptr) v += bias[gn];
      store_f(C, ci, v);
    }
  }
}

// xc = x - b_dec in the requested dtype (fp32 path of encode_pre).
template <typename XT, typename OT>
__global__ void sub_bias_kernel(const XT* __restrict__ x, const float* __restrict__ b,
                                OT* __restrict__ out, int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_f(out, i, __fsub_rn(load_f(x, i), b[i % cols]));
}

__global__ void exp_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = expf(in[i]);
}

// gate = float(pre > theta); feat = pre * gate (reference 860-883: the gate
// is the hard indicator plus a zero-valued bridge, promoted to fp32).
template <typename PT>
__global__ void jumprelu_fwd_kernel(const PT* __restrict__ pre, const float* __restrict__ log_thr,
                                    int64_t n_tokens, int64_t n_features, float* __restrict__ feat,
                                    float* __restrict__ gate) {
  const int64_t n = n_tokens * n_features;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t f = i % n_features;
    const float th = expf(log_thr[f]);
    const float p = load_f(pre, i);
    const float g = (p > th) ? 1.f : 0.f;
    if (gate != nullptr) gate[i] = g;
    if (feat != nullptr) feat[i] = p * g;
  }
}

// Straight-through backward, dense. Block = 32 features x 8 token lanes over
// a slab of JB_TOK tokens; per-feature partial sums land in part[slab, f].
constexpr int JB_TOK = 256;
template <typename PT>
__global__ void jumprelu_bwd_kernel(const PT* __restrict__ pre, const float* __restrict__ log_thr,
                                    int64_t n_tokens, int64_t n_features,
                                    const float* __restrict__ grad_feat,
                                    const float* __restrict__ grad_gate, float eps,
                                    PT* __restrict__ grad_pre, float* __restrict__ part) {
  __shared__ float s_sum[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t f = static_cast<int64_t>(blockIdx.x) * 32 + tx;
  const int64_t t0 = static_cast<int64_t>(blockIdx.y) * JB_TOK;
  float s = 0.f;
  if (f < n_features) {
    const float th = expf(log_thr[f]);
    for (int64_t t = t0 + ty; t < min(n_tokens, t0 + JB_TOK); t += 8) {
      const int64_t i = t * n_features + f;
      const float p = load_f(pre, i);
      const float gf = grad_feat != nullptr ? grad_feat[i] : 0.f;
      const float gg = grad_gate != nullptr ? grad_gate[i] : 0.f;
      const float gate = p > th ? 1.f : 0.f;
      if (grad_pre != nullptr) store_f(grad_pre, i, gf * gate);
      float comb = 0.f;
      if (grad_feat != nullptr) comb = __fmul_rn(p, gf);
      if (grad_gate != nullptr) comb = (grad_feat != nullptr) ? __fadd_rn(comb, gg) : gg;
      if (fabsf(__fsub_rn(p, th)) < eps) s += comb;
    }
  }
  s_sum[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && f < n_features) {
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += s_sum[k][tx];
    part[static_cast<size_t>(blockIdx.y) * n_features + f] = tot;
  }
}

__global__ void jumprelu_bwd_final_kernel(const float* __restrict__ part, int n_slabs,
                                          const float* __restrict__ log_thr, int64_t n_features,
                                          float eps, float* __restrict__ g_logthr) {
  for (int64_t f = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; f < n_features;
       f += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < n_slabs; ++k) s += part[static_cast<size_t>(k) * n_features + f];
    const float th = expf(log_thr[f]);
    g_logthr[f] += -(s / (eps + eps)) * th;
  }
}

template <typename XT>
__global__ void column_sum_kernel(const XT* __restrict__ X, int64_t rows, int64_t cols,
                                  float alpha, float beta, float* __restrict__ out) {
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < cols;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int64_t r = 0; r < rows; ++r) s += load_f(X, r * cols + c);
    out[c] = (beta != 0.f ? beta * out[c] : 0.f) + alpha * s;
  }
}

// One warp per row: norm, then divide (torch: W.div_(W.norm(...).clamp(min=1e-8))).
__global__ void renorm_rows_kernel(float* __restrict__ W, int64_t rows, int64_t cols,
                                   bf16* __restrict__ shadow) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    float* row = W + r * cols;
    float ss = 0.f;
    for (int64_t c = lane; c < cols; c += 32) ss = fmaf(row[c], row[c], ss);
    const float nrm = fmaxf(sqrtf(warp_sum(ss)), 1e-8f);
    for (int64_t c = lane; c < cols; c += 32) {
      const float v = __fdiv_rn(row[c], nrm);
      row[c] = v;
      if (shadow != nullptr) shadow[r * cols + c] = __float2bfloat16_rn(v);
    }
  }
}

__global__ void to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

// Dense activations for the dense backward: acts = pre where pre > theta.
// (feature-major [F, ldp] in and out)
__global__ void gated_pre_kernel(const bf16* __restrict__ pre, const float* __restrict__ theta,
                                 int64_t n_tokens, int64_t n_features, int64_t ldp,
                                 bf16* __restrict__ out) {
  const int64_t n = n_tokens * n_features;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t f = i / n_tokens, t = i - f * n_tokens;
    const size_t o = static_cast<size_t>(f) * ldp + t;
    const float p = __bfloat162float(pre[o]);
    out[o] = (p > theta[f]) ? pre[o] : __float2bfloat16_rn(0.f);
  }
}

}  // namespace sae
