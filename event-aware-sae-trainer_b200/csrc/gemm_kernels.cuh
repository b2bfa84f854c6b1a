// Plain products on the tcgen05 tile GEMM: an epilogue that writes
// C = alpha * A B^T + beta * C (+ bias) with bounds checks on both output
// dimensions, and the bf16 transpose that turns an operand stored with its
// contraction dimension outermost into the K-major layout TMA feeds to the
// tensor cores.
//
// Users: the dense weight-gradient fallback of the fused step (dW_enc =
// dpre^T xc and dW_dec = acts^T go, contraction over the tokens), and the
// bf16 GEMMs of the module API (decode, its gradients and the encoder's
// weight gradient under autocast).
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include "tile_gemm.cuh"

namespace sae {

// Epilogue of a row-guarded product: rows of D beyond `rows` and columns
// beyond `cols` are computed on TMA's zero fill and never stored. Each
// epilogue thread owns one output row and stores 32 consecutive columns per
// chunk (eight 16-byte stores for fp32, four for bf16 when `vec` is set).
struct StoreEpi {
  static constexpr int kAux = AUX_NONE;
  static constexpr bool kAuxFeatureMajor = false;
  static constexpr bool kRowGuard = true;
  void* c;                // output, row r at c + r * ldc (elements)
  int64_t ldc;
  int64_t rows, cols;
  float alpha, beta;      // beta == 0: C is never read
  const float* bias;      // optional: per column (bias_per_row 0) or per row (1)
  int bias_per_row;
  int c_bf16;             // output dtype: 1 bf16, 0 fp32
  int vec;                // 1: c and ldc allow 16-byte stores
  // per tile
  int64_t r, n0;
  bool row_ok;
  float rbias;

  __device__ __forceinline__ void begin_tile(int m_tile, int n_tile, int row, int, int, bf16*) {
    r = static_cast<int64_t>(m_tile) * TILE_M + row;
    n0 = static_cast<int64_t>(n_tile) * TILE_N;
    row_ok = r < rows;
    rbias = (bias != nullptr && bias_per_row && row_ok) ? bias[r] : 0.f;
  }
  __device__ __forceinline__ void begin_half(int) {}
  __device__ __forceinline__ void end_half(int) {}
  __device__ __forceinline__ float value(float acc, float old, int64_t n) const {
    float v = alpha * acc;
    if (beta != 0.f) v = fmaf(beta, old, v);
    if (bias != nullptr) v += bias_per_row ? rbias : bias[n];
    return v;
  }
  __device__ __forceinline__ void chunk(int col, const float (&v)[32]) {
    const int64_t n = n0 + col;
    if (!row_ok || n >= cols) return;
    if (c_bf16) {
      bf16* p = static_cast<bf16*>(c) + r * ldc + n;
      if (vec && n + 32 <= cols) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 old = make_uint4(0, 0, 0, 0);
          if (beta != 0.f) old = reinterpret_cast<const uint4*>(p)[q];
          const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&old);
          uint4 out;
          __nv_bfloat162* w2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 of = __bfloat1622float2(o2[j]);
            const int e = 8 * q + 2 * j;
            w2[j] = __floats2bfloat162_rn(value(v[e], of.x, n + e), value(v[e + 1], of.y, n + e + 1));
          }
          reinterpret_cast<uint4*>(p)[q] = out;
        }
      } else {
        const int m = static_cast<int>(cols - n < 32 ? cols - n : 32);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j < m) {
            const float old = beta != 0.f ? __bfloat162float(p[j]) : 0.f;
            p[j] = __float2bfloat16_rn(value(v[j], old, n + j));
          }
        }
      }
    } else {
      float* p = static_cast<float*>(c) + r * ldc + n;
      if (vec && n + 32 <= cols) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
          if (beta != 0.f) old = reinterpret_cast<const float4*>(p)[q];
          const int e = 4 * q;
          float4 out;
          out.x = value(v[e], old.x, n + e);
          out.y = value(v[e + 1], old.y, n + e + 1);
          out.z = value(v[e + 2], old.z, n + e + 2);
          out.w = value(v[e + 3], old.w, n + e + 3);
          reinterpret_cast<float4*>(p)[q] = out;
        }
      } else {
        const int m = static_cast<int>(cols - n < 32 ? cols - n : 32);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j < m) {
            const float old = beta != 0.f ? p[j] : 0.f;
            p[j] = value(v[j], old, n + j);
          }
        }
      }
    }
  }
  __device__ __forceinline__ void end_tile() {}
};

// dst[c, r] = src[r, c] (bf16) for r < rows, c < cols; src rows lds apart,
// dst rows ldd apart (elements). 64 x 64 tiles staged through shared memory,
// tiles taken grid-stride; `vec`: both layouts allow 16-byte accesses.
constexpr int TP_TILE = 64;
__global__ void __launch_bounds__(256)
    transpose_bf16_kernel(const bf16* __restrict__ src, int64_t rows, int64_t cols, int64_t lds,
                          bf16* __restrict__ dst, int64_t ldd, int vec) {
  __shared__ __align__(16) bf16 s[TP_TILE][TP_TILE + 8];
  const int64_t rt = (rows + TP_TILE - 1) / TP_TILE;
  const int64_t ct = (cols + TP_TILE - 1) / TP_TILE;
  for (int64_t tile = blockIdx.x; tile < rt * ct; tile += gridDim.x) {
    const int64_t r0 = (tile / ct) * TP_TILE, c0 = (tile % ct) * TP_TILE;
    // read 64 rows x 8 groups of 8 columns
    for (int i = threadIdx.x; i < TP_TILE * 8; i += blockDim.x) {
      const int rr = i >> 3, g = i & 7;
      const int64_t r = r0 + rr, c = c0 + 8 * g;
      if (vec && r < rows && c + 8 <= cols) {
        *reinterpret_cast<uint4*>(&s[rr][8 * g]) =
            *reinterpret_cast<const uint4*>(src + r * lds + c);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          s[rr][8 * g + j] = (r < rows && c + j < cols) ? src[r * lds + c + j]
                                                        : __float2bfloat16_rn(0.f);
      }
    }
    __syncthreads();
    // write 64 columns x 8 groups of 8 rows
    for (int i = threadIdx.x; i < TP_TILE * 8; i += blockDim.x) {
      const int cc = i >> 3, g = i & 7;
      const int64_t c = c0 + cc, r = r0 + 8 * g;
      if (c >= cols) continue;
      if (vec && r + 8 <= rows) {
        uint4 out;
        bf16* o = reinterpret_cast<bf16*>(&out);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = s[8 * g + j][cc];
        *reinterpret_cast<uint4*>(dst + c * ldd + r) = out;
      } else {
        for (int j = 0; j < 8 && r + j < rows; ++j) dst[c * ldd + r + j] = s[8 * g + j][cc];
      }
    }
    __syncthreads();
  }
}

}  // namespace sae
