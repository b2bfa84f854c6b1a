// The sampled backward with its row gathers pipelined through shared memory.
//
// Same arithmetic, same reduction order and same outputs as
// sampled_backward_kernel (step_kernels.cuh), which issues each chunk's go /
// xc row loads from registers and waits for them before the chunk's dot
// products: one chunk's rows in flight per block. Here one warp of the block
// is also the producer of a ring of R entry slots in shared memory: for every
// upcoming CSR entry it issues a bulk copy (cp.async.bulk, no tensor map, no
// multicast) of the entry's go row -- and, for an active entry, its xc row --
// into a free slot, completing on that slot's mbarrier. The consumers (all
// threads) wait on the slot's barrier and read the rows from shared memory,
// so up to R entries' rows are in flight per block, independently of the
// compute.
//
// The producer runs at the block's barriers: after a chunk's reduction
// barrier it refills the slots of the chunks every thread has finished, and
// at the end of a feature it claims the next features from the global
// counter (a queue of up to Q claimed features, so the ring runs ahead across
// feature boundaries). Entries are issued and consumed in the same order, so
// entry k sits in slot k % R and completes phase (k / R) & 1 of that slot's
// barrier.
//
// Waits are bounded (mbar_wait: 2 s of globaltimer); a wait that gives up
// sets SAE_ERR_DEVICE_TIMEOUT and the block's abort flag, every thread runs on
// to the next barrier, the block stops writing, waits (bounded) for the copies
// it issued and returns.
#pragma once
#include "step_kernels.cuh"

namespace sae {

constexpr int RING_Q = 8;   // claimed-feature queue

__device__ __forceinline__ void bulk_copy_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory bytes of a ring of `slots` entry slots at row width d
// (a go row and an xc row of d bf16 each per slot, plus its mbarrier).
__host__ __device__ constexpr size_t ring_smem_bytes(int d, int slots) {
  return static_cast<size_t>(slots) * (4 * static_cast<size_t>(d) + 8) + 16;
}

// Producer state, held identically by the 32 lanes of warp 0.
struct RingProducer {
  int issued;     // entries issued so far
  int claimed;    // features claimed so far (pushed to the queue)
  int qidx;       // queue index of the feature being issued (-1: none)
  int pos, end;   // its entries not issued yet
  bool done;      // the global counter is exhausted
};

// Issue copies for the upcoming entries while slots are free (entries below
// `freed` have been read by every thread), claiming features from the global
// counter when the one being issued is exhausted and the queue has room
// (`started`: features the consumers have begun). All 32 lanes of warp 0 call
// it together; lane 0 writes the queue and the flags.
__device__ __forceinline__ void ring_produce(RingProducer& p, int freed, int started, int R,
                                             int lane, int* s_fq, int* s_qtail, int* s_done,
                                             uint32_t* s_val, uint8_t* ring, uint64_t* full,
                                             int* counter, int n_seg, const int* col_offs,
                                             const int* csr_tok, const uint32_t* csr_val,
                                             const bf16* go, const bf16* xc, int n_tokens,
                                             int d) {
  const uint32_t row = static_cast<uint32_t>(2 * d);
  while (true) {
    if (p.pos == p.end) {
      if (p.qidx + 1 < p.claimed) {            // the next feature already claimed
        ++p.qidx;
        const int sg = s_fq[p.qidx % RING_Q];
        p.pos = col_offs[sg];
        p.end = col_offs[sg + 1];
        continue;
      }
      if (p.done || p.claimed - started >= RING_Q) return;
      int sg = 0;
      if (lane == 0) sg = atomicAdd(counter, 1);
      sg = __shfl_sync(0xffffffffu, sg, 0);
      if (sg >= n_seg) {
        p.done = true;
        if (lane == 0) *s_done = 1;
        return;
      }
      if (lane == 0) s_fq[p.claimed % RING_Q] = sg;
      ++p.claimed;
      if (lane == 0) *s_qtail = p.claimed;
      p.qidx = p.claimed - 1;
      p.pos = col_offs[sg];
      p.end = col_offs[sg + 1];
      continue;
    }
    const int free_slots = R - (p.issued - freed);
    if (free_slots <= 0) return;
    const int n = min(min(free_slots, p.end - p.pos), 32);
    if (lane < n) {
      const int q = p.pos + lane;
      const int slot = (p.issued + lane) % R;
      // (the clamp only guards the row reads; the fill writes tokens < n_tokens)
      const int t = min(max(csr_tok[q], 0), n_tokens - 1);
      const uint32_t v = csr_val[q];
      s_val[slot] = v;
      uint8_t* dst = ring + static_cast<size_t>(slot) * 2 * row;
      const bool act = (v & CSR_ACTIVE) != 0;
      mbar_arrive_expect_tx(&full[slot], act ? 2 * row : row);
      bulk_copy_g2s(dst, go + static_cast<size_t>(t) * d, row, &full[slot]);
      if (act) bulk_copy_g2s(dst + row, xc + static_cast<size_t>(t) * d, row, &full[slot]);
    }
    p.pos += n;
    p.issued += n;
  }
}

// Arguments and outputs as sampled_backward_kernel; R: ring slots (<= 32),
// dynamic shared memory ring_smem_bytes(d, R).
template <int C, int U, int MAX_THREADS, int MIN_BLOCKS>
__global__ void __launch_bounds__(MAX_THREADS, MIN_BLOCKS)
    sampled_backward_ring_kernel(const int* __restrict__ col_offs, const int* __restrict__ csr_tok,
                                 const uint32_t* __restrict__ csr_val, const bf16* __restrict__ go,
                                 const bf16* __restrict__ xc, const bf16* __restrict__ w_dec,
                                 const float* __restrict__ theta, int n_features, int n_tokens,
                                 int d, float eps, int accumulate, float* __restrict__ g_wdec,
                                 float* __restrict__ g_wenc, float* __restrict__ g_logthr,
                                 float* __restrict__ g_benc, float* __restrict__ db_enc,
                                 int* __restrict__ counter, const SaeB200StepStats* stats,
                                 const int* __restrict__ seg_rows, int honor_overflow,
                                 float* __restrict__ row_sumsq, int R) {
  if (honor_overflow && stats != nullptr && stats->csr_overflow) return;
  extern __shared__ __align__(128) uint8_t ring[];
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(R) * 4 * d);
  __shared__ uint32_t s_val[32];
  __shared__ int s_fq[RING_Q];
  __shared__ int s_qtail, s_done, s_abort;
  __shared__ float s_red[2][32][C];   // [chunk parity][warp][entry]
  const int tid = threadIdx.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  const int nvec = d / 8;
  const bool has = (tid + 1) * U <= nvec;
  const float gate_grad = stats != nullptr ? stats->gate_grad : 0.f;   // (band entries only)
  const size_t slot_bytes = static_cast<size_t>(4) * d;
  volatile int* abort_flag = &s_abort;
  if (tid == 0) {
    for (int s = 0; s < R; ++s) mbar_init(&full[s], 1);
    s_qtail = 0;
    s_done = 0;
    s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  RingProducer p{0, 0, -1, 0, 0, false};
  if (wid == 0)
    ring_produce(p, 0, 0, R, lane, s_fq, &s_qtail, &s_done, s_val, ring, full, counter,
                 n_features, col_offs, csr_tok, csr_val, go, xc, n_tokens, d);
  __syncthreads();
  int cons = 0, started = 0, par = 0;
  while (started < s_qtail && !*abort_flag) {
    const int sg = s_fq[started % RING_Q];
    ++started;
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
    for (int i0 = s; i0 < e; i0 += C) {
      const int n = min(C, e - i0);
      float part[C];
      uint32_t v[C];
#pragma unroll
      for (int r = 0; r < C; ++r) {
        part[r] = 0.f;
        v[r] = 0u;
        if (r < n) {
          const int k = cons + r;
          const int slot = k % R;
          mbar_wait(&full[slot], static_cast<uint32_t>((k / R) & 1), abort_flag);
          v[r] = s_val[slot];
          if (has) {
            const uint4* gs = reinterpret_cast<const uint4*>(ring + slot * slot_bytes) + U * tid;
            float a = 0.f;
#pragma unroll
            for (int u = 0; u < U; ++u) {
              float g8[8];
              unpack8(gs[u], g8);
#pragma unroll
              for (int j = 0; j < 8; ++j) a = fmaf(g8[j], wf[8 * u + j], a);
            }
            part[r] = a;
          }
        }
      }
      const float q = warp_sum_c<C>(part, lane);
      constexpr int kStride = 32 / C;
      if ((lane & (kStride - 1)) == 0) s_red[par][wid][lane / kStride] = q;
      __syncthreads();
      const bool ab = *abort_flag;
      // every thread is past the previous chunk: its slots may be refilled
      if (wid == 0 && !ab)
        ring_produce(p, cons, started, R, lane, s_fq, &s_qtail, &s_done, s_val, ring, full,
                     counter, n_features, col_offs, csr_tok, csr_val, go, xc, n_tokens, d);
#pragma unroll
      for (int r = 0; r < C; ++r) {
        if (r < n) {
          float a = 0.f;
          for (int w = 0; w < nw; ++w) a += s_red[par][w][r];
          const float gfv = bf16_round(a);
          const float pv = __uint_as_float(v[r] << 16);
          if (v[r] & CSR_ACTIVE) {
            if (has) {
              const uint8_t* sl = ring + ((cons + r) % R) * slot_bytes;
              const uint4* gs = reinterpret_cast<const uint4*>(sl) + U * tid;
              const uint4* xs = reinterpret_cast<const uint4*>(sl + 2 * d) + U * tid;
#pragma unroll
              for (int u = 0; u < U; ++u) {
                float g8[8], x8[8];
                unpack8(gs[u], g8);
                unpack8(xs[u], x8);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  ad[8 * u + j] = fmaf(pv, g8[j], ad[8 * u + j]);
                  ae[8 * u + j] = fmaf(gfv, x8[j], ae[8 * u + j]);
                }
              }
            }
            db += gfv;
          }
          if (v[r] & CSR_BAND) thr += __fadd_rn(__fmul_rn(pv, gfv), gate_grad);
        }
      }
      cons += n;
      par ^= 1;
      if (ab) break;
    }
    __syncthreads();   // every thread is done with this feature's slots
    if (!*abort_flag) {
      float sq = 0.f;
      if (has) {
        const size_t o = static_cast<size_t>(f) * d + static_cast<size_t>(tid) * 8 * U;
#pragma unroll
        for (int q4 = 0; q4 < 2 * U; ++q4) {
          if (g_wdec != nullptr) {
            float4* pw = reinterpret_cast<float4*>(g_wdec + o) + q4;
            float4 a4 = make_float4(ad[4 * q4], ad[4 * q4 + 1], ad[4 * q4 + 2], ad[4 * q4 + 3]);
            if (accumulate) {
              const float4 u4 = *pw;
              a4.x += u4.x; a4.y += u4.y; a4.z += u4.z; a4.w += u4.w;
            }
            *pw = a4;
            sq = fmaf(a4.x, a4.x, sq); sq = fmaf(a4.y, a4.y, sq);
            sq = fmaf(a4.z, a4.z, sq); sq = fmaf(a4.w, a4.w, sq);
          }
          float4* pe = reinterpret_cast<float4*>(g_wenc + o) + q4;
          float4 e4 = make_float4(ae[4 * q4], ae[4 * q4 + 1], ae[4 * q4 + 2], ae[4 * q4 + 3]);
          if (accumulate) {
            const float4 u4 = *pe;
            e4.x += u4.x; e4.y += u4.y; e4.z += u4.z; e4.w += u4.w;
          }
          *pe = e4;
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
      // the ring runs on into the next features (claims them if needed)
      if (wid == 0)
        ring_produce(p, cons, started, R, lane, s_fq, &s_qtail, &s_done, s_val, ring, full,
                     counter, n_features, col_offs, csr_tok, csr_val, go, xc, n_tokens, d);
    }
    __syncthreads();   // the queue and the flags the producer wrote are visible
  }
  // Every slot's last copy has landed before the block's shared memory goes
  // away (immediate unless the block aborted with copies in flight; a slot is
  // re-armed only after its previous entry was consumed, so its last issued
  // phase is the only one that can be pending).
  if (wid == 0 && lane == 0)
    for (int k = max(0, p.issued - R); k < p.issued; ++k)
      mbar_wait(&full[k % R], static_cast<uint32_t>((k / R) & 1), nullptr);
}

}  // namespace sae
