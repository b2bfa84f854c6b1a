/*
 * sae_b200.h -- C ABI of the B200 (sm_100a) JumpReLU sparse-autoencoder step.
 *
 * The library replaces the per-step SAE compute of the event-aware SAE trainer
 * (sae_trainer_rolling.py): encoder pre-activation with the JumpReLU gate,
 * decode + reconstruction loss, the backward pass with the straight-through
 * threshold estimator, global gradient clipping and the L2-decay Adam step
 * followed by decoder-column / encoder-row renormalisation.
 *
 * Conventions
 *  - Every pointer in a struct or argument is a DEVICE pointer unless noted.
 *  - All work is enqueued on the caller's stream; nothing here synchronises
 *    the device or allocates memory. Scratch comes from a caller-provided
 *    workspace sized by sae_b200_workspace_bytes().
 *  - Every entry point returns 0 (SAE_OK) or one of the SAE_ERR_* codes
 *    below; none throws or aborts. sae_b200_last_error() gives a message.
 *  - bf16 arrays are passed as void* (IEEE bfloat16, little-endian).
 *  - The decoder is stored feature-major: W_dec_fm[f, :] is decoder column f
 *    of the reference's W_dec.weight [d, F] (W_dec.weight == W_dec_fm^T).
 *
 * Citations are to the reference project's files (path:line).
 */
#ifndef SAE_B200_H
#define SAE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define SAE_OK 0
#define SAE_ERR_INVALID_ARGUMENT 1   /* null pointer, negative size, bad dtype */
#define SAE_ERR_UNSUPPORTED_SHAPE 2  /* shape outside what the kernels handle */
#define SAE_ERR_MISALIGNED 3         /* pointer / stride not 16-byte aligned */
#define SAE_ERR_WORKSPACE_TOO_SMALL 4
#define SAE_ERR_CSR_OVERFLOW 5       /* more CSR entries than csr_capacity */
#define SAE_ERR_CUDA 6               /* a CUDA runtime call failed */
#define SAE_ERR_DEVICE_TIMEOUT 7     /* a bounded device-side wait ran out */
#define SAE_ERR_NO_DEVICE 8

#define SAE_DTYPE_F32 0
#define SAE_DTYPE_BF16 1

/* Parameters of one JumpReLU SAE (reference: _JumpReLUSAE.__init__,
 * sae_trainer_rolling.py:772-800). */
typedef struct SaeB200Model {
  int64_t d_in;
  int64_t n_features;
  float* W_enc;          /* [F, d]  encoder weight (nn.Linear rows) */
  float* b_enc;          /* [F]     encoder bias */
  float* W_dec_fm;       /* [F, d]  decoder, feature-major */
  float* b_dec;          /* [d]     decoder bias / encoder pre-bias */
  float* log_threshold;  /* [F] */
  void* W_enc_bf16;      /* [F, d]  bf16 copy fed to the tensor cores */
  void* W_dec_bf16;      /* [F, d]  bf16 copy of W_dec_fm */
} SaeB200Model;

/* Gradients, same shapes and layouts as SaeB200Model's fp32 arrays. */
typedef struct SaeB200Grads {
  float* W_enc;
  float* b_enc;
  float* W_dec_fm;  /* may be NULL when the decoder is frozen */
  float* b_dec;
  float* log_threshold;
} SaeB200Grads;

/* One microbatch of the training step (reference loop body,
 * sae_trainer_rolling.py:2914-3016). */
typedef struct SaeB200StepConfig {
  int64_t n_tokens;        /* tokens in this microbatch (rows of x) */
  int64_t csr_capacity;    /* CSR entries the workspace holds: active (token, feature)
                              pairs, plus the inactive in-band pairs when sampled */
  float lambda_l0;         /* scheduler.lambda_l0 */
  float al_mu;             /* sae_cfg.al_mu */
  float target_l0;         /* sae_cfg.target_l0 */
  float ste_bandwidth;     /* sae.ste_bandwidth (epsilon of the STE band) */
  int32_t accum_steps;     /* microbatches per optimizer step */
  int32_t accumulate;      /* 0: gradients overwrite, 1: gradients add */
  int32_t train_decoder;   /* 0: frozen decoder (no W_dec gradient) */
  int32_t force_simt;      /* 1: CUDA-core tile GEMM even where tcgen05 applies */
  int32_t grad_feat_gemm;  /* backward: 0 = sampled grad_feat on the active and in-band
                              entries only (default); 1 = the dense tcgen05 grad_feat
                              GEMM with the STE epilogue. Same gradients; forward and
                              backward of a microbatch must use the same value. */
  int32_t pre_entries_only; /* forward, sampled backward only: 1 = store pre only in the
                              32-token words holding an active or in-band entry (all
                              that the decode and the sampled backward read); 0 = store
                              all of it, as sae_b200_train_backward_dense and
                              sae_b200_aux_forward need (they refuse a cfg with 1). */
} SaeB200StepConfig;

/* Step statistics, written on the device; copy back with one memcpy. */
typedef struct SaeB200StepStats {
  float recon_loss;     /* mean((x - x_hat)^2) / accum_steps        (2964-2965) */
  float l0;             /* mean active features per token            (2958,2969) */
  float sparsity_loss;  /* (lambda*s + mu/2*s^2)/accum, s = max(0, l0-target) */
  float gate_grad;      /* d loss / d gate element                             */
  float loss;           /* recon_loss + sparsity_loss                          */
  float grad_norm;      /* pre-clip global L2 norm of all gradients   (3049)   */
  float clip_coef;      /* min(1, max_norm / (grad_norm + 1e-6))               */
  int32_t nnz;          /* active (token, feature) pairs in this microbatch    */
  int32_t csr_overflow; /* 1 when csr_pairs > csr_capacity: use the dense backward */
  int32_t csr_pairs;    /* entries of the backward's CSR: nnz, plus the inactive
                           in-band pairs when the sampled backward is on      */
  float aux_loss;       /* dead-feature aux loss (2986-2998), 0 without it;
                           sae_b200_aux_forward also adds it to `loss`        */
  int32_t reserved[5];
} SaeB200StepStats;

/* Adam hyper-parameters for one parameter tensor. The five tensors are, in
 * order: W_enc, b_enc, W_dec_fm, b_dec, log_threshold (the reference's four
 * param groups, sae_trainer_rolling.py:2536-2541, flattened). */
typedef struct SaeB200AdamTensor {
  float lr, beta1, beta2, eps, weight_decay;
  float grad_scale;    /* host factor on the gradient (W_enc dampening, 3069-3074) */
  int32_t step;        /* Adam step count AFTER this update (>= 1) */
  int32_t use_clip;    /* 1: also multiply the gradient by stats->clip_coef */
  int32_t skip;        /* 1: leave this tensor untouched (frozen / no grad) */
  int32_t renorm_rows; /* 1: renormalise rows to unit L2 norm afterwards */
} SaeB200AdamTensor;

typedef struct SaeB200AdamState {
  float* exp_avg[5];
  float* exp_avg_sq[5];
} SaeB200AdamState;

/* ----------------------------------------------------------------- basics */
int sae_b200_version(void);
const char* sae_b200_last_error(void);
/* Reads (and optionally clears) the device status word that bounded waits
 * set when they give up. Synchronises the calling thread with the device. */
int sae_b200_get_device_status(int* status_out, int clear);

/* Number of kernels this library has launched in the process so far. */
int64_t sae_b200_launch_count(void);

/* Optional timing hook: while set, the library records start_event before and
 * stop_event after every launch of the chosen kernel on the launch stream
 * (cudaEvent_t handles owned by the caller; NULL, NULL clears it).
 * kernel: SAE_KERNEL_ENCODER_GEMM (tile GEMM of the forwards),
 * SAE_KERNEL_GRAD_GEMM (tile GEMM of the backwards, or the sampled backward),
 * SAE_KERNEL_DECODE (gathered decode of the forwards), SAE_KERNEL_ADAM (all
 * launches of one sae_b200_adam_step), SAE_KERNEL_EXCHANGE or
 * SAE_KERNEL_DENSE_WGRAD (below). */
#define SAE_KERNEL_ENCODER_GEMM 0
#define SAE_KERNEL_GRAD_GEMM 1
#define SAE_KERNEL_DECODE 2   /* the gathered decode of every forward */
#define SAE_KERNEL_ADAM 3     /* one optimizer update (Adam + renorm + bf16 copies) */
#define SAE_KERNEL_EXCHANGE 4 /* the NVLink peer exchange of sae_b200_shard_forward_p2p
                                 (both flag barriers and the cross-shard sum) */
#define SAE_KERNEL_DENSE_WGRAD 5 /* the dW_enc tile GEMM of the dense backward */
int sae_b200_set_kernel_timer(int kernel, void* start_event, void* stop_event);

/* Bytes of scratch the training step needs for up to max_tokens tokens. */
int sae_b200_workspace_bytes(int64_t max_tokens, int64_t d_in, int64_t n_features,
                             int64_t csr_capacity, size_t* bytes_out);

/* Byte offsets, inside the workspace of a step over n_tokens tokens, of the
 * intermediates a caller may inspect after sae_b200_train_forward/backward:
 * [0] theta f32 [F]        [1] xc bf16 [B, d]
 * [2] pre bf16, feature-major [F, ldp], ldp = sae_b200_pre_pitch(B)
 * [3] mask u32 [B, ceil(F/32)] (bit f%32 of word f/32: feature f active)
 * [4] go bf16 [B, d]       [5] per-token active count i32 [B]
 * [6] per-token squared error f32 [B]   [7] CSR row offsets i32 [F + 1]
 * [8] CSR token ids i32 [nnz]           [9] CSR values u32 [nnz]
 *     (low half: bf16 pre-activation, high half: bf16 gated grad_feat) */
#define SAE_WS_N_OFFSETS 10
/* Row pitch, in tokens, of the feature-major [F, ldp] pre-activation arrays:
 * n_tokens rounded up to a multiple of 64, plus 64, plus another 64 if that
 * is a power of two (a 2^k-byte pitch concentrates TMA boxes on few DRAM
 * channels). */
int64_t sae_b200_pre_pitch(int64_t n_tokens);
int sae_b200_workspace_offsets(int64_t n_tokens, int64_t d_in, int64_t n_features,
                               int64_t csr_capacity, size_t* offsets_out /* [10] */);

/* ------------------------------------------------------- fused hot path */
/* Forward of one microbatch: theta = exp(log_threshold); xc = x - b_dec;
 * pre = xc W_enc^T + b_enc (bf16, tcgen05); gate = pre > theta; active sets;
 * x_hat = gathered decode + b_dec; residual loss; sparsity term.
 * Replaces _EncoderPreBias.forward (sae_trainer_rolling.py:584-590),
 * _jumprelu_forward (827-901), decode/_SparseDecode.forward (922-950,
 * 628-637) and the loss lines 2954-2974.
 * x: [n_tokens, d] of x_dtype. x_hat_out: optional fp32 [n_tokens, d].
 * fired: [F] uint8, OR-accumulated (reference fired_accum, 3016). */
int sae_b200_train_forward(const SaeB200Model* model, const void* x, int x_dtype,
                           const SaeB200StepConfig* cfg, void* workspace,
                           size_t workspace_bytes, SaeB200StepStats* stats,
                           float* x_hat_out, uint8_t* fired, void* stream);

/* Backward of the microbatch last passed to sae_b200_train_forward (same
 * workspace): dense grad_feat GEMM with the STE epilogue, sparse scatter of
 * dW_enc / dW_dec over the active pairs, b_enc / b_dec / log_threshold
 * gradients. Replaces loss.backward() through _SparseDecode.backward
 * (639-654), the hooks 784-825 and _EncoderPreBias.backward (592-607).
 * When stats->csr_overflow is set on the device the sparse scatter is
 * skipped; the caller then runs sae_b200_train_backward_dense. With the
 * sampled backward (grad_feat_gemm = 0) an overflowed microbatch leaves every
 * gradient untouched, so the call may be queued before the host has read the
 * forward's statistics. */
int sae_b200_train_backward(const SaeB200Model* model, const SaeB200Grads* grads,
                            const SaeB200StepConfig* cfg, void* workspace,
                            size_t workspace_bytes, SaeB200StepStats* stats, void* stream);

/* After a forward with pre_entries_only = 1 whose CSR overflowed: re-runs its
 * encoder on the same workspace (the forward's xc and thresholds) and stores
 * all of pre, which sae_b200_train_backward_dense and the sharded dense path
 * read. Statistics, fired flags and CSR offsets are left as they are. No
 * counterpart in the reference (its autograd keeps the dense pre tensor). */
int sae_b200_store_full_pre(const SaeB200Model* model, const SaeB200StepConfig* cfg,
                            void* workspace, size_t workspace_bytes, void* stream);

/* Same gradients without the capacity limit, for microbatches whose active
 * set overflowed csr_capacity (the reference's dense autograd: dW_enc = dpre^T xc,
 * _EncoderPreBias.backward 592-607; dW_dec = acts^T go, decode 922-925). The two
 * weight-gradient contractions over the tokens run on the tcgen05 tile GEMM
 * (CUDA cores when cfg->force_simt is set). dense_scratch: device buffer owned
 * by the caller, 16-byte aligned, of at least sae_b200_dense_scratch_bytes()
 * bytes (the dense [F, ldp] operand and the transposed xc and go [d, ldp]);
 * smaller buffers return SAE_ERR_WORKSPACE_TOO_SMALL. */
int sae_b200_dense_scratch_bytes(int64_t n_tokens, int64_t d_in, int64_t n_features,
                                 size_t* bytes_out);
int sae_b200_train_backward_dense(const SaeB200Model* model, const SaeB200Grads* grads,
                                  const SaeB200StepConfig* cfg, void* workspace,
                                  size_t workspace_bytes, SaeB200StepStats* stats,
                                  void* dense_scratch, size_t dense_scratch_bytes, void* stream);

/* Global gradient norm and clip coefficient (torch.nn.utils.clip_grad_norm_,
 * called at sae_trainer_rolling.py:3049). Writes stats->grad_norm and
 * stats->clip_coef; the scaling itself is applied inside sae_b200_adam_step.
 * workspace: SAE_GRAD_NORM_WORKSPACE_BYTES of scratch (not the step workspace,
 * whose forward intermediates it would overwrite). */
#define SAE_GRAD_NORM_WORKSPACE_BYTES (592 * 4)
int sae_b200_grad_norm(const SaeB200Model* model, const SaeB200Grads* grads, float max_norm,
                       void* workspace, size_t workspace_bytes, SaeB200StepStats* stats,
                       void* stream);

/* The same norm and clip coefficient (clip_grad_norm_, 3049) straight after
 * sae_b200_train_backward with grad_feat_gemm = 0: the sampled backward leaves
 * per-feature sums of squares of the final W_enc, W_dec, b_enc and
 * log_threshold gradients in the step workspace, so this call reads those
 * F x warps partials and the b_dec gradient instead of all the gradients
 * again. Valid only when that backward ran to completion on these gradients
 * (no CSR overflow, no aux backward or other gradient edit since); otherwise
 * call sae_b200_grad_norm. cfg and workspace: those of the backward;
 * norm_workspace: SAE_GRAD_NORM_WORKSPACE_BYTES. */
int sae_b200_grad_norm_sampled(const SaeB200Model* model, const SaeB200Grads* grads,
                               const SaeB200StepConfig* cfg, const void* workspace,
                               size_t workspace_bytes, float max_norm, void* norm_workspace,
                               size_t norm_workspace_bytes, SaeB200StepStats* stats,
                               void* stream);

/* Inference: encoder GEMM + JumpReLU gate + gathered decode, no loss and no
 * backward state: x_hat_out [n_tokens, d] fp32 = bf16(gathered decoder sum) +
 * b_dec, the forward of the module (encode 910-912 + decode 922-950; also the
 * inference helper examples/use_trained_sae.py:58-75). active_counts_out
 * (optional, int32 [n_tokens]) gets each token's L0; fired (optional, uint8
 * [F]) is OR-accumulated. workspace: sae_b200_workspace_bytes(n_tokens, d, F, 0). */
int sae_b200_encode_decode(const SaeB200Model* model, const void* x, int x_dtype,
                           int64_t n_tokens, void* workspace, size_t workspace_bytes,
                           float* x_hat_out, int32_t* active_counts_out, uint8_t* fired,
                           void* stream);

/* ------------------------------------------------ dead-feature aux loss
 * The trainer's aux reconstruction for features silent for AUX_DEAD_THRESHOLD
 * steps (sae_trainer_rolling.py:2986-2998; helper 252-293): per token, the
 * top-k of relu(pre[:, dead]) reconstruct the detached residual through their
 * decoder columns, aux = coeff * mean((x - x_hat - x_aux)^2) / accum. Ties at
 * the k-th value go to the lower dead-list index. Call sae_b200_aux_forward
 * after sae_b200_train_forward (same workspace, which still holds pre; x_hat:
 * the fp32 x_hat_out of that forward) and before reading the stats;
 * sae_b200_aux_backward after sae_b200_train_backward(_dense): it adds the aux
 * gradients of the dead features' W_enc rows, b_enc, W_dec rows and the b_dec
 * term. Not available on a dictionary shard (the top-k spans all shards). */
typedef struct SaeB200AuxConfig {
  const int32_t* dead;  /* [n_dead] device array of feature ids in [0, F), ascending */
  int64_t n_dead;
  int32_t k;            /* eff_k = min(aux_k, n_dead), >= 1 */
  float coeff;          /* AUX_COEFF (1/32) */
} SaeB200AuxConfig;
int sae_b200_aux_workspace_bytes(int64_t max_tokens, int64_t d_in, int64_t n_features,
                                 int64_t max_dead, int32_t k, size_t* bytes_out);
int sae_b200_aux_forward(const SaeB200Model* model, const void* x, int x_dtype,
                         const float* x_hat, const SaeB200StepConfig* cfg, void* workspace,
                         size_t workspace_bytes, const SaeB200AuxConfig* aux, void* aux_workspace,
                         size_t aux_workspace_bytes, SaeB200StepStats* stats, void* stream);
int sae_b200_aux_backward(const SaeB200Model* model, const SaeB200Grads* grads,
                          const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                          const SaeB200AuxConfig* aux, void* aux_workspace,
                          size_t aux_workspace_bytes, void* stream);

/* ------------------------------------------- dictionary-sharded wide SAE
 * One wide SAE with its dictionary split over GPUs: each rank holds features
 * [r*F/N, (r+1)*F/N) (W_enc rows, b_enc, W_dec columns, log_threshold, their
 * gradients and Adam state); x and b_dec are replicated. The reference trains
 * the whole dictionary on one device; these entry points split the same step
 * (sae_trainer_rolling.py:2914-3090) at its three cross-feature sums, which the
 * caller adds over the ranks (e.g. an NCCL all-reduce on the same stream):
 *   1. sae_b200_shard_forward writes `exchange` = this shard's fp32 decoder
 *      sums [n_tokens, d] followed by its per-token active counts [n_tokens]
 *      (as floats); all-reduce(SUM) it, then sae_b200_shard_finish_forward
 *      forms x_hat = bf16(sum) + b_dec, the residual, loss, L0 and go (the
 *      same on every rank).
 *   2. sae_b200_shard_backward (shard_rank 0 owns the replicated b_dec term):
 *      all-reduce(SUM) grads->b_dec afterwards.
 *   3. sae_b200_grad_sumsq (pass b_dec's gradient on rank 0 only, NULL
 *      elsewhere): all-reduce(SUM) the float, then sae_b200_clip_from_sumsq.
 * The Adam step is local (b_dec's update is identical on every rank). With
 * N = 1 the sequence gives the same result as the unsharded entry points up
 * to fp32 summation order. */
int64_t sae_b200_shard_exchange_floats(int64_t n_tokens, int64_t d_in);

/* NVLink peer exchange (alternative to the all-reduce of step 1): every rank's
 * "peer buffer" -- [step workspace | exchange | flags] -- is mapped into every
 * rank by CUDA IPC, and sae_b200_shard_forward_p2p does sae_b200_shard_forward,
 * the cross-shard sum and sae_b200_shard_finish_forward in one call: rank r
 * sums the partials of tokens [rB/N, (r+1)B/N) with peer loads and writes
 * their go, squared error and count into every rank's workspace with peer
 * stores, between two flag barriers (bounded: a barrier that waits over 2 s
 * sets SAE_ERR_DEVICE_TIMEOUT in the device status word and returns). The
 * backward and the two remaining scalar/vector sums are as above. Setup-time
 * calls only: sae_b200_peer_alloc is the one entry point that allocates
 * (cudaMalloc of the buffer, zero-filled); free it after every rank is done. */
#define SAE_MAX_PEERS 8
#define SAE_PEER_HANDLE_BYTES 64
typedef struct SaeB200Peers {
  int32_t rank, world;     /* world <= SAE_MAX_PEERS, one GPU per rank */
  uint32_t epoch;          /* larger than any epoch used before with these buffers */
  int32_t reserved;
  uint64_t exchange_offset, flags_offset;   /* from sae_b200_peer_buffer_bytes */
  void* base[SAE_MAX_PEERS];                /* rank p's buffer, mapped here (own included) */
} SaeB200Peers;
int sae_b200_peer_buffer_bytes(int64_t max_tokens, int64_t d_in, int64_t n_features,
                               int64_t csr_capacity, size_t* bytes_out,
                               uint64_t* exchange_offset_out, uint64_t* flags_offset_out);
int sae_b200_peer_alloc(size_t bytes, void** ptr_out, void* handle_out /* 64 bytes, host */);
int sae_b200_peer_open(const void* handle /* host */, void** ptr_out);
int sae_b200_peer_close(void* ptr);
int sae_b200_peer_free(void* ptr);
int sae_b200_shard_forward_p2p(const SaeB200Model* model, const void* x, int x_dtype,
                               const SaeB200StepConfig* cfg, const SaeB200Peers* peers,
                               SaeB200StepStats* stats, uint8_t* fired, void* stream);
/* Encoder GEMM + gate + CSR offsets + gathered decode of this shard's features
 * (decode / _SparseDecode.forward 922-950 restricted to the shard). */
int sae_b200_shard_forward(const SaeB200Model* model, const void* x, int x_dtype,
                           const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                           SaeB200StepStats* stats, uint8_t* fired, float* exchange,
                           void* stream);
/* Residual, reconstruction loss, sparsity term and go from the summed
 * exchange (loss lines 2963-2974). */
int sae_b200_shard_finish_forward(const SaeB200Model* model, const void* x, int x_dtype,
                                  const SaeB200StepConfig* cfg, void* workspace,
                                  size_t workspace_bytes, SaeB200StepStats* stats,
                                  const float* exchange, float* x_hat_out, void* stream);
/* sae_b200_train_backward (dense_scratch NULL) or _dense (dense_scratch set)
 * of this shard; on shard_rank != 0 the b_dec gradient is overwritten with the
 * shard's encoder term -(sum_b dpre) W_enc_shard only (601), so that the sum
 * over ranks is the full gradient, accumulated once. */
int sae_b200_shard_backward(const SaeB200Model* model, const SaeB200Grads* grads,
                            const SaeB200StepConfig* cfg, void* workspace, size_t workspace_bytes,
                            SaeB200StepStats* stats, int shard_rank, void* dense_scratch,
                            size_t dense_scratch_bytes, void* stream);
/* *sumsq_out (device float) = sum of squares of the non-NULL gradients. */
/* The same shard sum of squares straight after a sampled sae_b200_shard_backward
 * that did not overflow (and after the b_dec all-reduce): from the backward's
 * per-feature partials of the W_enc, W_dec, b_enc and log_threshold gradient
 * rows plus grads->b_dec (pass NULL on the ranks that do not count the
 * replicated b_dec), without another pass over the gradients. cfg, workspace:
 * those of the backward; norm_workspace: SAE_GRAD_NORM_WORKSPACE_BYTES. */
int sae_b200_grad_sumsq_sampled(const SaeB200Model* model, const SaeB200Grads* grads,
                                const SaeB200StepConfig* cfg, const void* workspace,
                                size_t workspace_bytes, void* norm_workspace,
                                size_t norm_workspace_bytes, float* sumsq_out, void* stream);
int sae_b200_grad_sumsq(const SaeB200Model* model, const SaeB200Grads* grads, void* workspace,
                        size_t workspace_bytes, float* sumsq_out, void* stream);
/* stats->grad_norm = sqrt(*sumsq), stats->clip_coef = min(1, max_norm/(norm+1e-6))
 * (clip_grad_norm_, 3049). */
int sae_b200_clip_from_sumsq(const float* sumsq, float max_norm, SaeB200StepStats* stats,
                             void* stream);

/* L2-decay Adam (torch.optim.Adam, sae_trainer_rolling.py:2536-2541, 3076)
 * fused with the decoder-column / encoder-row renormalisation (778-782,
 * 3086-3090) and the refresh of the bf16 weight copies. */
int sae_b200_adam_step(const SaeB200Model* model, const SaeB200Grads* grads,
                       const SaeB200AdamState* state, const SaeB200AdamTensor* hyper /*[5], host*/,
                       const SaeB200StepStats* stats, void* stream);

/* ------------------------------------------ dense pieces of the module API */
/* pre = (x - b_dec) W_enc^T + b_enc. pre_dtype BF16: computed the autocast way
 * (bf16 operands, fp32 accumulate, bf16 result) on the tile GEMM. pre_dtype
 * F32: fp32 throughout. xc_out (optional, pre_dtype): the saved x - b_dec.
 * Replaces _EncoderPreBias.forward / _pre (567-590, 903-908). */
int sae_b200_encode_pre(const SaeB200Model* model, const void* x, int x_dtype, int64_t n_tokens,
                        void* pre_out, int pre_dtype, void* xc_out, int force_simt,
                        void* workspace, size_t workspace_bytes, void* stream);

/* gate = 1[pre > exp(log_threshold)], feat = pre * gate (fp32 outputs).
 * Replaces the forward of _jumprelu_forward (827-901). */
int sae_b200_jumprelu_forward(const void* pre, int pre_dtype, const float* log_threshold,
                              int64_t n_tokens, int64_t n_features, float* feat_out,
                              float* gate_out, void* stream);

/* Straight-through backward of the JumpReLU (hooks 784-825 / _JumpReLUWithGate
 * 700-731): grad_pre = grad_feat * gate; combined = pre * grad_feat + grad_gate;
 * grad_log_threshold += -sum_t where(|pre - theta| < eps, combined) / (2 eps) * theta.
 * grad_feat / grad_gate may be NULL (treated as zero); grad_pre_out may be NULL.
 * n_tokens <= 65535 * 256 (one grid row per 256-token slab); larger calls
 * return SAE_ERR_UNSUPPORTED_SHAPE. */
int sae_b200_jumprelu_backward(const void* pre, int pre_dtype, const float* log_threshold,
                               int64_t n_tokens, int64_t n_features, const float* grad_feat,
                               const float* grad_gate, float eps, void* grad_pre_out,
                               float* grad_log_threshold, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Allocation-free variant of sae_b200_jumprelu_backward. (No counterpart in
 * the reference trainer; it exists for callers of this library.)
 * Some callers cannot hand the library a workspace: a host framework that has
 * already reserved the GPU's memory for its own caching allocator (so that an
 * extra cudaMalloc would fail or fragment it), or a latency-critical caller
 * that must not make the implicitly synchronising cudaMalloc/cudaFree calls.
 * This entry point takes the same inputs and outputs but keeps its scratch --
 * the per-slab partial sums of the threshold gradient -- in a fixed array of
 * SAE_JUMPRELU_BWD_STATIC_FLOATS floats (4 MiB) compiled into the library, so
 * it allocates nothing. Every GPU that loads the library holds that array
 * until the process exits.
 *  - Limit: ceil(n_tokens / 256) * n_features must not exceed
 *    SAE_JUMPRELU_BWD_STATIC_FLOATS (e.g. 65536 tokens x 4096 features);
 *    larger calls return SAE_ERR_UNSUPPORTED_SHAPE and do nothing, as do
 *    calls with more than 65535 * 256 tokens (one grid row per slab).
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress, with that device current); make that first call
 *    before capturing any stream into a CUDA graph.
 *  - All calls share the one array, and each call overwrites the part it
 *    reads before reading it. Calls that can run at the same time on the GPU
 *    (different streams without ordering, or several host threads) race on
 *    the array and give wrong results; order them on one stream. */
#define SAE_JUMPRELU_BWD_STATIC_FLOATS (1 << 20)
int sae_b200_jumprelu_backward_static(const void* pre, int pre_dtype, const float* log_threshold,
                                      int64_t n_tokens, int64_t n_features,
                                      const float* grad_feat, const float* grad_gate, float eps,
                                      void* grad_pre_out, float* grad_log_threshold, void* stream);

/* General strided product: C = alpha * A B^T + beta * C (+ bias[n]).
 * A[m, k] at A + m*sam + k*sak; B[n, k] at B + n*sbn + k*sbk; C[m, n] at
 * C + m*scm + n*scn (strides in elements). beta == 0 never reads C.
 * bf16 A and B stored K-major (sak == sbk == 1, 16-byte aligned bases, sam and
 * sbn multiples of 8), M, N >= 128, K >= 64 and an output with scn == 1 or
 * scm == 1 run on the tcgen05 tile GEMM (fp32 accumulate); everything else, and
 * every call while SAE_B200_GEMM_SIMT=1 is set in the environment, on CUDA cores
 * in fp32. The module API's dense products under bf16 autocast: decode
 * (sae_trainer_rolling.py:922-925) and the weight / input gradients of the
 * decoder and encoder (592-607). */
int sae_b200_gemm(int64_t M, int64_t N, int64_t K, float alpha, const void* A, int a_dtype,
                  int64_t sam, int64_t sak, const void* B, int b_dtype, int64_t sbn,
                  int64_t sbk, float beta, void* C, int c_dtype, int64_t scm, int64_t scn,
                  const float* bias_n, void* stream);

/* dst[c, r] = src[r, c] for a bf16 [rows, cols] matrix with rows lds apart into
 * [cols, rows] with rows ldd apart (elements): puts an operand whose
 * contraction dimension is outermost into the K-major layout sae_b200_gemm
 * feeds to the tensor cores. No counterpart in the reference (cuBLAS takes
 * either layout). */
int sae_b200_transpose(const void* src, int dtype, int64_t rows, int64_t cols, int64_t lds,
                       void* dst, int64_t ldd, void* stream);

/* out[c] = beta * out[c] + alpha * sum_r X[r, c]  (X row-major [rows, cols]). */
int sae_b200_column_sum(const void* X, int x_dtype, int64_t rows, int64_t cols, float alpha,
                        float beta, float* out, void* stream);

/* Rows of W [rows, cols] to unit L2 norm (norm clamped at 1e-8), optionally
 * refreshing a bf16 copy. Replaces _normalize_decoder (778-782) on the
 * feature-major decoder and the W_enc row renorm (3089-3090). */
int sae_b200_renorm_rows(float* W, int64_t rows, int64_t cols, void* shadow_bf16, void* stream);

/* dst (bf16) = src (fp32), n elements: refresh of a bf16 weight copy. */
int sae_b200_refresh_shadow(const float* src, void* dst_bf16, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SAE_B200_H */
