"""The reference's own training function driven with the B200 class installed.

sae_b200.install(T) makes the reference trainer construct B200JumpReLUSAE
(sae_trainer_rolling.py:553-562, _make_sae 961-966); train_sae_on_activations
(2382-3672) then runs its unchanged loop -- preflight probe, b_dec estimate,
autocast forward, loss.backward(), clip, dampening, its own torch Adam, renorms,
scheduler, revival bookkeeping, checkpoint writes -- on the library's module
API. A few steps on a small synthetic provider must finish with finite losses,
write the reference's state_dict keys and shapes, and launch this library's
kernels.

Needs the reference checkout (named by $SAE_REFERENCE_DIR) and a GPU in the
same place; skipped otherwise.
"""
import importlib
import math
import os
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF = os.environ.get("SAE_REFERENCE_DIR")
D, F, TOKENS, MB = 256, 2048, 2048, 1024

if not REF or not (Path(REF) / "sae_trainer_rolling.py").exists():
    pytest.skip("set SAE_REFERENCE_DIR to a checkout of the reference trainer",
                allow_module_level=True)


class _Provider:
    """The provider interface the trainer calls (next_batch, next_batch_to_device,
    get_state, restore_state, close): seeded superposition batches on the GPU."""

    def __init__(self):
        import sae_b200
        self.i = 0
        self.make = lambda s: sae_b200.superposition_batch(TOKENS, D, F, 16, math.log(8.0), 0.3,
                                                           seed=s, device=torch.device("cuda"))

    def next_batch(self):
        self.i += 1
        return self.make(100 + self.i)

    def next_batch_to_device(self, non_blocking=True):
        return self.next_batch()

    def get_state(self):
        return {"i": self.i}

    def restore_state(self, state):
        self.i = int(state.get("i", 0))

    def close(self):
        pass


@pytest.fixture(scope="module")
def trained(tmp_path_factory):
    out = tmp_path_factory.mktemp("ref_trainer")
    env = {"SAE_BATCH_TOKENS": str(TOKENS), "SAE_MICROBATCH_TOKENS": str(MB),
           "SAE_DATA_DIR": str(out)}
    old = {k: os.environ.get(k) for k in list(env) + ["WANDB_PROJECT", "SAE_HUB_ID"]}
    os.environ.update(env)
    os.environ.pop("WANDB_PROJECT", None)
    os.environ.pop("SAE_HUB_ID", None)
    sys.path.insert(0, REF)
    try:
        sys.modules.pop("sae_trainer_rolling", None)
        T = importlib.import_module("sae_trainer_rolling")
        import sae_b200
        from sae_b200 import _lib as L
        sae_b200.install(T)
        T.N_FEATURES = F
        launches0 = L.launch_count()
        metrics = T.train_sae_on_activations(20, D, 0, _Provider(), max_steps=3, bdec_batches=2,
                                             microbatch_tokens=MB, push=False)
        torch.cuda.synchronize()
        saved = sorted(Path(T.SAE_DIR).glob("layer_20_s0*/sae.pt"))
        return dict(T=T, metrics=metrics, launches=L.launch_count() - launches0, saved=saved)
    finally:
        sys.path.remove(REF)
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def test_training_finishes_with_finite_losses(trained):
    m = trained["metrics"]
    assert m, "the trainer returned no metrics"
    for key in ("recon_loss", "mean_l0"):
        if m.get(key) is not None:
            assert math.isfinite(float(m[key])), key


def test_checkpoint_has_the_reference_layout(trained):
    assert trained["saved"], "no sae.pt written"
    sd = torch.load(trained["saved"][-1], map_location="cpu")
    assert {"W_enc.weight", "W_enc.bias", "W_dec.weight", "b_dec", "log_threshold"} <= set(sd)
    assert tuple(sd["W_enc.weight"].shape) == (F, D)
    assert tuple(sd["W_dec.weight"].shape) == (D, F)
    assert torch.isfinite(sd["W_dec.weight"]).all()
    torch.testing.assert_close(sd["W_dec.weight"].float().norm(dim=0), torch.ones(F),
                               rtol=0, atol=1e-4)


def test_library_kernels_ran(trained):
    assert trained["launches"] > 0
