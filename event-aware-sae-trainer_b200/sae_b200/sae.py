"""JumpReLU SAE module with the reference trainer's API, computed by libsae_b200.

``B200JumpReLUSAE`` is a drop-in for ``_JumpReLUSAE``
(sae_trainer_rolling.py:753-958): the same constructor ``(d_in, n_features)``,
the same bit-identical initialisation from the torch RNG, the same parameter
names, shapes and ``state_dict`` keys (``W_enc.weight [F, d]``, ``W_enc.bias``,
``W_dec.weight [d, F]``, ``b_dec``, ``log_threshold``), the mutable
``ste_bandwidth`` and the methods ``encode``, ``encode_pre``, ``_pre``,
``apply_jumprelu``, ``l0_indicator``, ``jumprelu_with_gate``, ``decode``,
``forward`` and ``_normalize_decoder``. Assigning it to
``sae_trainer_rolling.JumpReLUSAE`` makes ``_make_sae`` build it
(``_ensure_sae_classes`` returns the global when it is set, 553-562).

Storage is B200-first: the decoder lives feature-major ``[F, d]`` (so a
feature's decoder row is contiguous for the gathered decode and the row
renormalisation) and ``W_dec.weight`` is the ``[d, F]`` transposed view of it;
bf16 copies of both weight matrices feed the tensor cores and are refreshed
whenever the fp32 weights change.

Every computation runs in the CUDA library; the module refuses CPU tensors.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn as nn

from . import _lib as L

INIT_THRESHOLD = 0.1   # sae_trainer_rolling.py:212
STE_BANDWIDTH = 0.1    # sae_trainer_rolling.py:232
# The reference reassociates the b_dec gradient whenever x needs no grad
# (SAE_FAST_PREBIAS, sae_trainer_rolling.py:178); the library always does.
_SHADOW_MODE = os.environ.get("SAE_B200_SHADOW_REFRESH", "auto").lower()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("B200JumpReLUSAE computes on CUDA devices only "
                               "(move the module and its inputs with .to('cuda'))")


def _dt_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return L.DTYPE_F32
    if t.dtype == torch.bfloat16:
        return L.DTYPE_BF16
    raise TypeError(f"sae_b200 kernels take float32 or bfloat16 tensors, got {t.dtype}")


def _autocast_bf16(device: torch.device) -> bool:
    return (device.type == "cuda" and torch.is_autocast_enabled("cuda")
            and torch.get_autocast_dtype("cuda") == torch.bfloat16)


_GEMM_SIMT = os.environ.get("SAE_B200_GEMM_SIMT", "0") == "1"


def _k_major(T: torch.Tensor, s_outer: int, s_k: int, n_outer: int, K: int):
    """A bf16 GEMM operand with its contraction dimension contiguous, as
    (tensor, outer stride, k stride): operands stored the other way round
    ([K, n_outer] rows s_k apart) are transposed by the library into a fresh
    [n_outer, K] buffer whose rows are padded to 16 bytes."""
    if s_k == 1 or s_outer != 1:
        return T, s_outer, s_k
    kp = (K + 7) // 8 * 8
    out = torch.empty(n_outer, kp, device=T.device, dtype=torch.bfloat16)
    L.call("sae_b200_transpose", L.ptr(T), L.DTYPE_BF16, K, n_outer, s_k, L.ptr(out), kp,
           _stream())
    return out, kp, 1


def gemm(M, N, K, A, sam, sak, B, sbn, sbk, C, scm, scn, *, alpha=1.0, beta=0.0, bias=None):
    """C = alpha A B^T + beta C (+ bias), arbitrary strides (elements). bf16
    products large enough for the tensor cores get K-major operands (see
    _k_major) and run on the tcgen05 tile GEMM; the rest on CUDA cores."""
    if (not _GEMM_SIMT and A.dtype == torch.bfloat16 and B.dtype == torch.bfloat16
            and M >= 128 and N >= 128 and K >= 64 and (scn == 1 or scm == 1)):
        A, sam, sak = _k_major(A, sam, sak, M, K)
        B, sbn, sbk = _k_major(B, sbn, sbk, N, K)
    L.call("sae_b200_gemm", M, N, K, alpha, L.ptr(A), _dt_code(A), sam, sak, L.ptr(B),
           _dt_code(B), sbn, sbk, beta, L.ptr(C), _dt_code(C), scm, scn, L.ptr(bias), _stream())


def column_sum(X: torch.Tensor, out: torch.Tensor, alpha=1.0, beta=0.0) -> torch.Tensor:
    X = X.contiguous()
    L.call("sae_b200_column_sum", L.ptr(X), _dt_code(X), X.shape[0], X.shape[1], alpha, beta,
           L.ptr(out), _stream())
    return out


def to_bf16(src: torch.Tensor, dst: Optional[torch.Tensor] = None) -> torch.Tensor:
    src = src.contiguous()
    if dst is None:
        dst = torch.empty(src.shape, device=src.device, dtype=torch.bfloat16)
    L.call("sae_b200_refresh_shadow", L.ptr(src), L.ptr(dst), src.numel(), _stream())
    return dst


class _Linear(nn.Module):
    """Parameter holder with nn.Linear's attribute names (weight [out, in], bias)."""

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor]):
        super().__init__()
        self.weight = nn.Parameter(weight)
        if bias is not None:
            self.bias = nn.Parameter(bias)
        else:
            self.register_parameter("bias", None)

    @property
    def in_features(self) -> int:
        return self.weight.shape[1]

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    def forward(self, x):
        # y = x W^T + b, on the library's strided GEMM.
        _require_cuda(x, self.weight)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        w = self.weight
        out = torch.empty(x2.shape[0], w.shape[0], device=x.device, dtype=torch.float32)
        gemm(x2.shape[0], w.shape[0], w.shape[1], x2, x2.stride(0), x2.stride(1), w, w.stride(0),
             w.stride(1), out, out.stride(0), out.stride(1),
             bias=None if self.bias is None else self.bias.detach())
        return out.reshape(*lead, w.shape[0])


# ---------------------------------------------------------------- autograd
class _EncoderPre(torch.autograd.Function):
    """pre = (x - b_dec) W_enc^T + b_enc with the reassociated b_dec gradient
    (_EncoderPreBias, sae_trainer_rolling.py:567-607). Under bf16 autocast the
    operands are bf16 and pre is bf16, as autocast's addmm produces."""

    @staticmethod
    def forward(ctx, x, weight, b_enc, b_dec, sae):
        x = x.contiguous()
        B = x.shape[0]
        bf = _autocast_bf16(x.device)
        model = sae._model_struct(need_shadows=bf)
        if bf:
            pre = torch.empty(B, sae.n_features, device=x.device, dtype=torch.bfloat16)
            xc = torch.empty(B, sae.d_in, device=x.device, dtype=torch.bfloat16)
            w_used = sae._shadow_enc
        else:
            pre = torch.empty(B, sae.n_features, device=x.device, dtype=torch.float32)
            xc = torch.empty(B, sae.d_in, device=x.device, dtype=torch.float32)
            w_used = weight.detach()
        L.call("sae_b200_encode_pre", model, L.ptr(x), _dt_code(x), B, L.ptr(pre), _dt_code(pre),
               L.ptr(xc), 0, None, 0, _stream())
        ctx.save_for_backward(xc, w_used)
        ctx.param_dtypes = (weight.dtype, b_enc.dtype, b_dec.dtype)
        return pre

    @staticmethod
    def backward(ctx, dpre):
        xc, w = ctx.saved_tensors
        dpre = dpre.contiguous()
        B, F = dpre.shape
        d = xc.shape[1]
        dev = dpre.device
        dW = torch.empty(F, d, device=dev, dtype=torch.float32)
        gemm(F, d, B, dpre, 1, F, xc, 1, d, dW, d, 1)                  # dpre^T xc
        db_enc = torch.empty(F, device=dev, dtype=torch.float32)
        column_sum(dpre, db_enc)                                        # sum_b dpre
        db_dec = torch.empty(1, d, device=dev, dtype=torch.float32)
        gemm(1, d, F, db_enc, F, 1, w, 1, d, db_dec, d, 1, alpha=-1.0)  # -(sum dpre) W
        return None, dW, db_enc, db_dec.reshape(d), None


class _JumpReLU(torch.autograd.Function):
    """(feat, gate) = (pre * 1[pre > θ], 1[pre > θ]) with the straight-through
    threshold gradient of _log_threshold_hook (sae_trainer_rolling.py:792-825):
    dlogθ = -Σ_b where(|pre - θ| < ε, pre * grad_feat + grad_gate) / (2ε) * θ,
    and grad_pre = grad_feat * gate. ε is read from the module at backward
    time, as the hook does."""

    @staticmethod
    def forward(ctx, pre, log_threshold, sae):
        pre = pre.contiguous()
        B, F = pre.shape
        feat = torch.empty(B, F, device=pre.device, dtype=torch.float32)
        gate = torch.empty(B, F, device=pre.device, dtype=torch.float32)
        L.call("sae_b200_jumprelu_forward", L.ptr(pre), _dt_code(pre),
               L.ptr(log_threshold.detach()), B, F, L.ptr(feat), L.ptr(gate), _stream())
        ctx.save_for_backward(pre, log_threshold)
        ctx.sae = sae
        return feat, gate

    @staticmethod
    def backward(ctx, grad_feat, grad_gate):
        pre, log_thr = ctx.saved_tensors
        B, F = pre.shape
        gf = None if grad_feat is None else grad_feat.float().contiguous()
        gg = None if grad_gate is None else grad_gate.float().contiguous()
        grad_pre = torch.empty_like(pre) if ctx.needs_input_grad[0] else None
        g_lt = torch.zeros(F, device=pre.device, dtype=torch.float32)
        slabs = (B + 255) // 256
        ws = torch.empty(slabs * F, device=pre.device, dtype=torch.float32)
        L.call("sae_b200_jumprelu_backward", L.ptr(pre), _dt_code(pre), L.ptr(log_thr.detach()),
               B, F, L.ptr(gf), L.ptr(gg), float(ctx.sae.ste_bandwidth), L.ptr(grad_pre),
               L.ptr(g_lt), L.ptr(ws), ws.numel() * 4, _stream())
        return grad_pre, g_lt.to(log_thr.dtype), None


class _Decode(torch.autograd.Function):
    """x_hat = acts W_dec^T + b_dec (decode, sae_trainer_rolling.py:922-925).
    Under bf16 autocast the GEMM takes bf16 operands and returns a bf16 result
    that is then added to the fp32 bias, as autocast's linear does. The weight
    gradient is produced feature-major and handed back as the [d, F] view."""

    @staticmethod
    def forward(ctx, acts, w_dec_view, b_dec, sae):
        acts = acts.contiguous()
        B, F = acts.shape
        d = sae.d_in
        bf = _autocast_bf16(acts.device)
        fm = sae._dec_fm()
        if bf:
            sae._model_struct(need_shadows=True)
            a_in = to_bf16(acts.float()) if acts.dtype != torch.bfloat16 else acts
            w_in = sae._shadow_dec
            tmp = torch.empty(B, d, device=acts.device, dtype=torch.bfloat16)
            gemm(B, d, F, a_in, F, 1, w_in, 1, d, tmp, d, 1)
            out = torch.empty(B, d, device=acts.device, dtype=torch.float32)
            gemm(B, d, 0, a_in, F, 1, w_in, 1, d, out, d, 1, beta=0.0, bias=b_dec.detach())
            out.add_(tmp.float())
        else:
            a_in, w_in = acts, fm.detach()
            out = torch.empty(B, d, device=acts.device, dtype=torch.float32)
            gemm(B, d, F, a_in, F, 1, w_in, 1, d, out, d, 1, bias=b_dec.detach())
        ctx.save_for_backward(a_in, w_in)
        ctx.bf = bf
        return out

    @staticmethod
    def backward(ctx, go):
        a_in, w_in = ctx.saved_tensors
        go = go.contiguous().float()
        B, d = go.shape
        F = a_in.shape[1]
        g_in = to_bf16(go) if ctx.bf else go
        grad_acts = None
        if ctx.needs_input_grad[0]:
            ga = torch.empty(B, F, device=go.device,
                             dtype=torch.bfloat16 if ctx.bf else torch.float32)
            gemm(B, F, d, g_in, d, 1, w_in, d, 1, ga, F, 1)             # go W_dec
            grad_acts = ga.float()
        grad_w = None
        if ctx.needs_input_grad[1]:
            g_fm = torch.empty(F, d, device=go.device, dtype=torch.float32)
            gemm(F, d, B, a_in, 1, F, g_in, 1, d, g_fm, d, 1)           # acts^T go
            grad_w = g_fm.t()
        grad_b = None
        if ctx.needs_input_grad[2]:
            grad_b = column_sum(go, torch.empty(d, device=go.device, dtype=torch.float32))
        return grad_acts, grad_w, grad_b, None


# ------------------------------------------------------------------ module
class B200JumpReLUSAE(nn.Module):
    """JumpReLU SAE on B200; see the module docstring for the contract."""

    def __init__(self, d_in: int, n_features: int, *, _tensors=None):
        super().__init__()
        self.d_in = int(d_in)
        self.n_features = int(n_features)
        if _tensors is None:
            # Same RNG draws as the reference constructor (772-800): two nn.Linear
            # initialisations, then orthogonal_ on the [d, F] decoder, unit
            # columns, W_enc = W_dec^T, b_enc = 0.
            enc = nn.Linear(d_in, n_features, bias=True)
            dec = nn.Linear(n_features, d_in, bias=False)
            with torch.no_grad():
                nn.init.orthogonal_(dec.weight)
                norms = dec.weight.norm(dim=0, keepdim=True).clamp(min=1e-8)
                dec.weight.div_(norms)
                enc.weight.copy_(dec.weight.t())
                enc.bias.zero_()
            w_enc = enc.weight.detach().clone()
            b_enc = enc.bias.detach().clone()
            dec_fm = dec.weight.detach().t().contiguous()      # [F, d] feature-major
            b_dec = torch.zeros(d_in)
            log_thr = torch.full((n_features,), math.log(INIT_THRESHOLD))
        else:
            w_enc, b_enc, dec_fm, b_dec, log_thr = _tensors
        self.W_enc = _Linear(w_enc, b_enc)
        self.W_dec = _Linear(dec_fm.t(), None)                 # [d, F] view
        self.b_dec = nn.Parameter(b_dec)
        self.log_threshold = nn.Parameter(log_thr)
        self.ste_bandwidth = STE_BANDWIDTH
        self._sparse_decode_calls = 0
        self._sparse_decode_fallbacks = 0
        self._shadow_enc: Optional[torch.Tensor] = None
        self._shadow_dec: Optional[torch.Tensor] = None
        self._shadow_key = None
        self._shadow_dirty = True
        self._state_probe = None   # callable returning optimizer-state versions

    # ---------------------------------------------------------- storage
    def _dec_fm(self) -> torch.Tensor:
        """The feature-major decoder storage [F, d] (W_dec.weight^T)."""
        w = self.W_dec.weight
        fm = w.t()
        if not fm.is_contiguous():
            # Someone replaced W_dec.weight with a [d, F]-contiguous tensor
            # (e.g. `.data = ...`): move it back to feature-major storage.
            with torch.no_grad():
                w.data = fm.contiguous().t()
            fm = w.t()
            self._shadow_dirty = True
        return fm

    def mark_weights_dirty(self) -> None:
        """Call after writing W_enc / W_dec through ``.data``: the bf16 copies
        the tensor cores read are rebuilt before the next computation."""
        self._shadow_dirty = True

    def _weights_key(self):
        key = [self.W_enc.weight._version, self.W_enc.weight.data_ptr(),
               self.W_dec.weight._version, self.W_dec.weight.data_ptr()]
        if self._state_probe is not None:
            key.extend(self._state_probe())
        return tuple(key)

    def _refresh_shadows(self, force: bool = False) -> None:
        fm = self._dec_fm()
        dev = fm.device
        if self._shadow_enc is None or self._shadow_enc.device != dev:
            self._shadow_enc = torch.empty(self.n_features, self.d_in, device=dev,
                                           dtype=torch.bfloat16)
            self._shadow_dec = torch.empty(self.n_features, self.d_in, device=dev,
                                           dtype=torch.bfloat16)
            force = True
        key = self._weights_key()
        if force or self._shadow_dirty or _SHADOW_MODE == "always" or key != self._shadow_key:
            to_bf16(self.W_enc.weight.detach(), self._shadow_enc)
            to_bf16(fm.detach(), self._shadow_dec)
            self._shadow_key = self._weights_key()
            self._shadow_dirty = False

    def _shadows_written(self) -> None:
        """The library just wrote fresh bf16 copies (fused Adam step)."""
        self._shadow_key = self._weights_key()
        self._shadow_dirty = False

    def _model_struct(self, need_shadows: bool = True) -> L.Model:
        _require_cuda(self.W_enc.weight)
        fm = self._dec_fm()
        for p in (self.W_enc.weight, self.W_enc.bias, self.b_dec, self.log_threshold):
            if p.dtype != torch.float32 or not p.is_contiguous():
                raise TypeError("B200JumpReLUSAE parameters must be contiguous float32")
        if fm.dtype != torch.float32:
            raise TypeError("B200JumpReLUSAE parameters must be float32")
        if need_shadows:
            self._refresh_shadows()
        return L.Model(self.d_in, self.n_features, L.ptr(self.W_enc.weight), L.ptr(self.W_enc.bias),
                       L.ptr(fm), L.ptr(self.b_dec), L.ptr(self.log_threshold),
                       L.ptr(self._shadow_enc) if need_shadows else 0,
                       L.ptr(self._shadow_dec) if need_shadows else 0)

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        res = super().load_state_dict(state_dict, strict=strict, assign=assign)
        self._shadow_dirty = True
        return res

    def _apply(self, fn, recurse=True):
        out = super()._apply(fn, recurse)
        self._shadow_enc = self._shadow_dec = None
        self._shadow_dirty = True
        return out

    # ---------------------------------------------------------- API
    def _normalize_decoder(self):
        """Unit-norm decoder columns (778-782): rows of the feature-major storage."""
        fm = self._dec_fm()
        _require_cuda(fm)
        with torch.no_grad():
            L.call("sae_b200_renorm_rows", L.ptr(fm), self.n_features, self.d_in, None, _stream())
        self._shadow_dirty = True

    def _pre(self, x: torch.Tensor) -> torch.Tensor:
        """Encoder pre-activation (903-908); the reassociated Function unless x
        needs a gradient, in which case the plain x W^T path runs."""
        _require_cuda(x)
        if not x.requires_grad:
            # Under no_grad this is the same forward (bf16 tile GEMM under
            # autocast) without the autograd record.
            return _EncoderPre.apply(x, self.W_enc.weight, self.W_enc.bias, self.b_dec, self)
        xc = x - self.b_dec
        pre = _PlainLinear.apply(xc, self.W_enc.weight, self.W_enc.bias)
        return pre.to(torch.bfloat16) if _autocast_bf16(x.device) else pre

    def encode_pre(self, x):
        return self._pre(x)

    def _jumprelu_forward(self, pre, need_gate: bool):
        _require_cuda(pre)
        feat, gate = _JumpReLU.apply(pre, self.log_threshold, self)
        return (feat, gate) if need_gate else feat

    def encode(self, x, k: int = 0):
        return self._jumprelu_forward(self._pre(x), need_gate=False)

    def apply_jumprelu(self, pre):
        return self._jumprelu_forward(pre, need_gate=False)

    def l0_indicator(self, pre):
        _, gate = self._jumprelu_forward(pre, need_gate=True)
        return gate

    def jumprelu_with_gate(self, pre):
        return self._jumprelu_forward(pre, need_gate=True)

    def decode(self, acts, active_max: Optional[int] = None):
        _require_cuda(acts)
        if acts.dim() != 2:
            lead = acts.shape[:-1]
            return self.decode(acts.reshape(-1, acts.shape[-1]), active_max).reshape(*lead, self.d_in)
        return _Decode.apply(acts, self.W_dec.weight, self.b_dec, self)

    def forward(self, x, k: int = 0):
        acts = self.encode(x, k=k)
        x_hat = self.decode(acts)
        return x_hat, acts

    @torch.no_grad()
    def reconstruct(self, x: torch.Tensor, fired: Optional[torch.Tensor] = None):
        """Inference without the dense [B, F] activations: one library call runs
        the encoder GEMM with the JumpReLU gate and the gathered decode
        (bf16 operands and pre-activations, fp32 accumulation -- the autocast
        forward). Returns (x_hat fp32 [B, d], per-token L0 int32 [B]);
        ``fired`` (uint8 [F]) is OR-accumulated when given."""
        _require_cuda(x)
        if x.dim() != 2 or x.shape[1] != self.d_in:
            raise ValueError(f"x must be [tokens, {self.d_in}]")
        if x.dtype not in (torch.bfloat16, torch.float32):
            x = x.float()
        x = x.contiguous()
        B = x.shape[0]
        model = self._model_struct(need_shadows=True)
        need = L.workspace_bytes(B, self.d_in, self.n_features, 0)
        ws = getattr(self, "_infer_ws", None)
        if ws is None or ws.numel() < need or ws.device != x.device:
            ws = self._infer_ws = torch.empty(need, device=x.device, dtype=torch.uint8)
        x_hat = torch.empty(B, self.d_in, device=x.device, dtype=torch.float32)
        counts = torch.empty(B, device=x.device, dtype=torch.int32)
        L.call("sae_b200_encode_decode", model, L.ptr(x), _dt_code(x), B, L.ptr(ws), ws.numel(),
               L.ptr(x_hat), L.ptr(counts), L.ptr(fired), _stream())
        return x_hat, counts


class _PlainLinear(torch.autograd.Function):
    """y = x W^T + b with gradients for x as well (the reference's fallback when
    x requires grad, 908)."""

    @staticmethod
    def forward(ctx, x, w, b):
        x2 = x.float().contiguous()
        B, d = x2.shape
        F = w.shape[0]
        out = torch.empty(B, F, device=x.device, dtype=torch.float32)
        gemm(B, F, d, x2, d, 1, w.detach(), w.stride(0), w.stride(1), out, F, 1, bias=b.detach())
        ctx.save_for_backward(x2, w)
        return out

    @staticmethod
    def backward(ctx, g):
        x2, w = ctx.saved_tensors
        g = g.float().contiguous()
        B, F = g.shape
        d = x2.shape[1]
        gx = torch.empty(B, d, device=g.device, dtype=torch.float32)
        gemm(B, d, F, g, F, 1, w.detach(), w.stride(1), w.stride(0), gx, d, 1)
        gw = torch.empty(F, d, device=g.device, dtype=torch.float32)
        gemm(F, d, B, g, 1, F, x2, 1, d, gw, d, 1)
        gb = column_sum(g, torch.empty(F, device=g.device, dtype=torch.float32))
        return gx, gw, gb


def sae_from_tensors(W_enc: torch.Tensor, b_enc: torch.Tensor, W_dec_fm: torch.Tensor,
                     b_dec: torch.Tensor, log_threshold: torch.Tensor) -> B200JumpReLUSAE:
    """A module over existing float32 tensors (no initialisation, no RNG use):
    W_enc [F, d], b_enc [F], the feature-major decoder W_dec_fm [F, d] (row f
    is decoder column f), b_dec [d], log_threshold [F]."""
    F, d = W_enc.shape
    if W_dec_fm.shape != (F, d) or b_enc.shape != (F,) or b_dec.shape != (d,) \
            or log_threshold.shape != (F,):
        raise ValueError("inconsistent SAE tensor shapes")
    ts = tuple(t.detach().float().contiguous().clone()
               for t in (W_enc, b_enc, W_dec_fm, b_dec, log_threshold))
    return B200JumpReLUSAE(d, F, _tensors=ts)


def make_sae(d_in: int, n_features: int, seed: int = 0) -> B200JumpReLUSAE:
    """``_make_sae`` (sae_trainer_rolling.py:961-966): seed, then construct."""
    torch.manual_seed(seed)
    return B200JumpReLUSAE(d_in, n_features)


def install(reference_module) -> None:
    """Make the reference trainer build this class: sets its JumpReLUSAE global,
    which _ensure_sae_classes returns as-is (sae_trainer_rolling.py:553-562)."""
    reference_module.JumpReLUSAE = B200JumpReLUSAE
