"""ctypes binding of libsae_b200.so (the C ABI declared in include/sae_b200.h).

Every call goes through ``call()``, which raises ``SaeB200Error`` with the
library's message when an entry point returns a non-zero status. The library
is loaded from this package directory; importing it on a machine without the
built ``.so`` raises immediately -- there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_uint8, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsae_b200.so")

SAE_OK = 0
SAE_ERR_INVALID_ARGUMENT = 1
SAE_ERR_UNSUPPORTED_SHAPE = 2
SAE_ERR_MISALIGNED = 3
SAE_ERR_WORKSPACE_TOO_SMALL = 4
SAE_ERR_CSR_OVERFLOW = 5
SAE_ERR_CUDA = 6
SAE_ERR_DEVICE_TIMEOUT = 7
SAE_ERR_NO_DEVICE = 8

GRAD_NORM_WORKSPACE_BYTES = 592 * 4
JUMPRELU_BWD_STATIC_FLOATS = 1 << 20   # scratch size of sae_b200_jumprelu_backward_static

DTYPE_F32 = 0
DTYPE_BF16 = 1


class SaeB200Error(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"sae_b200 error {code}: {message}")
        self.code = code


class Model(ctypes.Structure):
    _fields_ = [
        ("d_in", c_int64),
        ("n_features", c_int64),
        ("W_enc", c_void_p),
        ("b_enc", c_void_p),
        ("W_dec_fm", c_void_p),
        ("b_dec", c_void_p),
        ("log_threshold", c_void_p),
        ("W_enc_bf16", c_void_p),
        ("W_dec_bf16", c_void_p),
    ]


class Grads(ctypes.Structure):
    _fields_ = [
        ("W_enc", c_void_p),
        ("b_enc", c_void_p),
        ("W_dec_fm", c_void_p),
        ("b_dec", c_void_p),
        ("log_threshold", c_void_p),
    ]


class StepConfig(ctypes.Structure):
    _fields_ = [
        ("n_tokens", c_int64),
        ("csr_capacity", c_int64),
        ("lambda_l0", c_float),
        ("al_mu", c_float),
        ("target_l0", c_float),
        ("ste_bandwidth", c_float),
        ("accum_steps", c_int32),
        ("accumulate", c_int32),
        ("train_decoder", c_int32),
        ("force_simt", c_int32),
        ("grad_feat_gemm", c_int32),
        ("pre_entries_only", c_int32),
    ]


class StepStats(ctypes.Structure):
    _fields_ = [
        ("recon_loss", c_float),
        ("l0", c_float),
        ("sparsity_loss", c_float),
        ("gate_grad", c_float),
        ("loss", c_float),
        ("grad_norm", c_float),
        ("clip_coef", c_float),
        ("nnz", c_int32),
        ("csr_overflow", c_int32),
        ("csr_pairs", c_int32),
        ("aux_loss", c_float),
        ("reserved", c_int32 * 5),
    ]


STATS_FLOATS = ctypes.sizeof(StepStats) // 4
STATS_FIELDS = [name for name, _ in StepStats._fields_ if name != "reserved"]


class AuxConfig(ctypes.Structure):
    _fields_ = [
        ("dead", c_void_p),
        ("n_dead", c_int64),
        ("k", c_int32),
        ("coeff", c_float),
    ]


MAX_PEERS = 8
PEER_HANDLE_BYTES = 64


class Peers(ctypes.Structure):
    _fields_ = [
        ("rank", c_int32),
        ("world", c_int32),
        ("epoch", ctypes.c_uint32),
        ("reserved", c_int32),
        ("exchange_offset", ctypes.c_uint64),
        ("flags_offset", ctypes.c_uint64),
        ("base", c_void_p * MAX_PEERS),
    ]


class AdamTensor(ctypes.Structure):
    _fields_ = [
        ("lr", c_float),
        ("beta1", c_float),
        ("beta2", c_float),
        ("eps", c_float),
        ("weight_decay", c_float),
        ("grad_scale", c_float),
        ("step", c_int32),
        ("use_clip", c_int32),
        ("skip", c_int32),
        ("renorm_rows", c_int32),
    ]


class AdamState(ctypes.Structure):
    _fields_ = [("exp_avg", c_void_p * 5), ("exp_avg_sq", c_void_p * 5)]


_SIGNATURES = {
    "sae_b200_version": ([], c_int),
    "sae_b200_last_error": ([], ctypes.c_char_p),
    "sae_b200_get_device_status": ([POINTER(c_int), c_int], c_int),
    "sae_b200_launch_count": ([], c_int64),
    "sae_b200_pre_pitch": ([c_int64], c_int64),
    "sae_b200_set_kernel_timer": ([c_int, c_void_p, c_void_p], c_int),
    "sae_b200_workspace_bytes": ([c_int64, c_int64, c_int64, c_int64, POINTER(c_size_t)], c_int),
    "sae_b200_workspace_offsets": ([c_int64, c_int64, c_int64, c_int64, POINTER(c_size_t)], c_int),
    "sae_b200_train_forward": (
        [POINTER(Model), c_void_p, c_int, POINTER(StepConfig), c_void_p, c_size_t, c_void_p,
         c_void_p, c_void_p, c_void_p], c_int),
    "sae_b200_train_backward": (
        [POINTER(Model), POINTER(Grads), POINTER(StepConfig), c_void_p, c_size_t, c_void_p,
         c_void_p], c_int),
    "sae_b200_store_full_pre": (
        [POINTER(Model), POINTER(StepConfig), c_void_p, c_size_t, c_void_p], c_int),
    "sae_b200_dense_scratch_bytes": ([c_int64, c_int64, c_int64, POINTER(c_size_t)], c_int),
    "sae_b200_train_backward_dense": (
        [POINTER(Model), POINTER(Grads), POINTER(StepConfig), c_void_p, c_size_t, c_void_p,
         c_void_p, c_size_t, c_void_p], c_int),
    "sae_b200_encode_decode": (
        [POINTER(Model), c_void_p, c_int, c_int64, c_void_p, c_size_t, c_void_p, c_void_p,
         c_void_p, c_void_p], c_int),
    "sae_b200_aux_workspace_bytes": (
        [c_int64, c_int64, c_int64, c_int64, c_int32, POINTER(c_size_t)], c_int),
    "sae_b200_aux_forward": (
        [POINTER(Model), c_void_p, c_int, c_void_p, POINTER(StepConfig), c_void_p, c_size_t,
         POINTER(AuxConfig), c_void_p, c_size_t, c_void_p, c_void_p], c_int),
    "sae_b200_aux_backward": (
        [POINTER(Model), POINTER(Grads), POINTER(StepConfig), c_void_p, c_size_t,
         POINTER(AuxConfig), c_void_p, c_size_t, c_void_p], c_int),
    "sae_b200_shard_exchange_floats": ([c_int64, c_int64], c_int64),
    "sae_b200_peer_buffer_bytes": (
        [c_int64, c_int64, c_int64, c_int64, POINTER(c_size_t), POINTER(ctypes.c_uint64),
         POINTER(ctypes.c_uint64)], c_int),
    "sae_b200_peer_alloc": ([c_size_t, POINTER(c_void_p), c_void_p], c_int),
    "sae_b200_peer_open": ([c_void_p, POINTER(c_void_p)], c_int),
    "sae_b200_peer_close": ([c_void_p], c_int),
    "sae_b200_peer_free": ([c_void_p], c_int),
    "sae_b200_shard_forward_p2p": (
        [POINTER(Model), c_void_p, c_int, POINTER(StepConfig), POINTER(Peers), c_void_p, c_void_p,
         c_void_p], c_int),
    "sae_b200_shard_forward": (
        [POINTER(Model), c_void_p, c_int, POINTER(StepConfig), c_void_p, c_size_t, c_void_p,
         c_void_p, c_void_p, c_void_p], c_int),
    "sae_b200_shard_finish_forward": (
        [POINTER(Model), c_void_p, c_int, POINTER(StepConfig), c_void_p, c_size_t, c_void_p,
         c_void_p, c_void_p, c_void_p], c_int),
    "sae_b200_shard_backward": (
        [POINTER(Model), POINTER(Grads), POINTER(StepConfig), c_void_p, c_size_t, c_void_p, c_int,
         c_void_p, c_size_t, c_void_p], c_int),
    "sae_b200_grad_sumsq_sampled": (
        [POINTER(Model), POINTER(Grads), POINTER(StepConfig), c_void_p, c_size_t, c_void_p,
         c_size_t, c_void_p, c_void_p], c_int),
    "sae_b200_grad_sumsq": (
        [POINTER(Model), POINTER(Grads), c_void_p, c_size_t, c_void_p, c_void_p], c_int),
    "sae_b200_clip_from_sumsq": ([c_void_p, c_float, c_void_p, c_void_p], c_int),
    "sae_b200_grad_norm": (
        [POINTER(Model), POINTER(Grads), c_float, c_void_p, c_size_t, c_void_p, c_void_p], c_int),
    "sae_b200_grad_norm_sampled": (
        [POINTER(Model), POINTER(Grads), POINTER(StepConfig), c_void_p, c_size_t, c_float,
         c_void_p, c_size_t, c_void_p, c_void_p], c_int),
    "sae_b200_adam_step": (
        [POINTER(Model), POINTER(Grads), POINTER(AdamState), POINTER(AdamTensor), c_void_p,
         c_void_p], c_int),
    "sae_b200_encode_pre": (
        [POINTER(Model), c_void_p, c_int, c_int64, c_void_p, c_int, c_void_p, c_int, c_void_p,
         c_size_t, c_void_p], c_int),
    "sae_b200_jumprelu_forward": (
        [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p], c_int),
    "sae_b200_jumprelu_backward": (
        [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_float, c_void_p,
         c_void_p, c_void_p, c_size_t, c_void_p], c_int),
    "sae_b200_jumprelu_backward_static": (
        [c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_float, c_void_p,
         c_void_p, c_void_p], c_int),
    "sae_b200_gemm": (
        [c_int64, c_int64, c_int64, c_float, c_void_p, c_int, c_int64, c_int64, c_void_p, c_int,
         c_int64, c_int64, c_float, c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p], c_int),
    "sae_b200_transpose": (
        [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p], c_int),
    "sae_b200_column_sum": (
        [c_void_p, c_int, c_int64, c_int64, c_float, c_float, c_void_p, c_void_p], c_int),
    "sae_b200_renorm_rows": ([c_void_p, c_int64, c_int64, c_void_p, c_void_p], c_int),
    "sae_b200_refresh_shadow": ([c_void_p, c_void_p, c_int64, c_void_p], c_int),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C event-aware-sae-trainer_b200/csrc` "
            "(or __graft_entry__.build()). There is no non-CUDA implementation.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (argtypes, restype) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = lib
    return lib


def exported_symbols() -> list:
    return list(_SIGNATURES)


def call(name: str, *args) -> None:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != SAE_OK:
        msg = lib.sae_b200_last_error()
        raise SaeB200Error(rc, msg.decode() if msg else name)


KERNEL_ENCODER_GEMM = 0
KERNEL_GRAD_GEMM = 1
KERNEL_DECODE = 2
KERNEL_ADAM = 3
KERNEL_EXCHANGE = 4
KERNEL_DENSE_WGRAD = 5


def pre_pitch(n_tokens: int) -> int:
    """Row pitch (tokens) of the feature-major [F, ldp] pre-activation arrays."""
    return int(load().sae_b200_pre_pitch(n_tokens))


def launch_count() -> int:
    return int(load().sae_b200_launch_count())


def set_kernel_timer(kernel: int, start_event=None, stop_event=None) -> None:
    """Record torch.cuda.Event pairs around the chosen kernel's launches."""
    for ev in (start_event, stop_event):
        # torch creates the CUDA event on its first record: make sure it exists
        if ev is not None and ev.cuda_event == 0:
            ev.record()
    s = 0 if start_event is None else start_event.cuda_event
    e = 0 if stop_event is None else stop_event.cuda_event
    call("sae_b200_set_kernel_timer", kernel, s, e)


def device_status(clear: bool = True) -> int:
    lib = load()
    out = c_int(0)
    call("sae_b200_get_device_status", ctypes.byref(out), 1 if clear else 0)
    return out.value


def aux_workspace_bytes(max_tokens: int, d_in: int, n_features: int, max_dead: int,
                        k: int) -> int:
    out = c_size_t(0)
    call("sae_b200_aux_workspace_bytes", max_tokens, d_in, n_features, max_dead, k,
         ctypes.byref(out))
    return out.value


def dense_scratch_bytes(n_tokens: int, d_in: int, n_features: int) -> int:
    """Bytes of the caller's scratch for the dense weight-gradient backward."""
    out = c_size_t(0)
    call("sae_b200_dense_scratch_bytes", n_tokens, d_in, n_features, ctypes.byref(out))
    return out.value


def workspace_bytes(max_tokens: int, d_in: int, n_features: int, csr_capacity: int) -> int:
    out = c_size_t(0)
    call("sae_b200_workspace_bytes", max_tokens, d_in, n_features, csr_capacity, ctypes.byref(out))
    return out.value


WS_REGIONS = ("theta", "xc", "pre", "mask", "go", "tok_cnt", "tok_sqerr", "col_offs", "csr_tok",
              "csr_val")


def workspace_offsets(n_tokens: int, d_in: int, n_features: int, csr_capacity: int) -> dict:
    out = (c_size_t * len(WS_REGIONS))()
    call("sae_b200_workspace_offsets", n_tokens, d_in, n_features, csr_capacity, out)
    return dict(zip(WS_REGIONS, list(out)))


def ptr(t) -> int:
    """Device address of a tensor (None -> NULL)."""
    return 0 if t is None else t.data_ptr()
