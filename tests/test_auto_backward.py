"""FusedStep(grad_feat="auto"): the choice between the sampled backward and
the dense grad_feat GEMM, from the previous microbatch's statistics (host
logic only; the two backwards themselves are parity-tested on the GPU)."""
from sae_b200.step import FusedStep


def _fs(threshold=100.0):
    fs = FusedStep.__new__(FusedStep)        # the decision needs no device state
    fs.grad_feat_mode = "auto"
    fs.grad_feat = "sampled"
    fs.auto_threshold = threshold
    fs._band_ratio = 1.0
    return fs


def _st(pairs, nnz, overflow=0):
    return {"csr_pairs": pairs, "nnz": nnz, "csr_overflow": overflow}


def test_switches_to_gemm_above_the_threshold_and_back_with_hysteresis():
    fs = _fs(100.0)
    fs._auto_update(_st(90 * 1000, 60 * 1000), 1000)     # 90 entries / token
    assert fs.grad_feat == "sampled"
    fs._auto_update(_st(150 * 1000, 100 * 1000), 1000)   # 150: above
    assert fs.grad_feat == "gemm" and fs._band_ratio == 1.5
    fs._auto_update(_st(100 * 1000, 60 * 1000), 1000)    # GEMM mode: 60 active x 1.5 = 90
    assert fs.grad_feat == "gemm"                          # inside the 20% band
    fs._auto_update(_st(70 * 1000, 50 * 1000), 1000)     # 50 x 1.5 = 75 < 80
    assert fs.grad_feat == "sampled"


def test_overflow_and_fixed_modes_do_not_switch():
    fs = _fs(100.0)
    fs._auto_update(_st(900 * 1000, 800 * 1000, overflow=1), 1000)
    assert fs.grad_feat == "sampled"
    fs.grad_feat_mode = "sampled"
    fs._auto_update(_st(900 * 1000, 800 * 1000), 1000)
    assert fs.grad_feat == "sampled"
