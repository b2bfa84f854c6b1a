"""B200-native JumpReLU SAE training step (sm_100a CUDA behind a C ABI).

Public API:
  B200JumpReLUSAE, make_sae, install   -- the reference SAE module's API
  B200Adam, FusedStep                  -- optimizer and the fused training step
  ShardedFusedStep, shard_sae,
  make_shard_sae                       -- one wide SAE split over GPUs by features
  DeviceActivationPool                 -- a layer's activation pool resident in HBM
  superposition_batch                  -- the benchmark's synthetic activations
"""
from ._lib import SaeB200Error, load as load_library  # noqa: F401
from .sae import B200JumpReLUSAE, install, make_sae  # noqa: F401
from .step import B200Adam, FusedStep, reference_param_groups  # noqa: F401
from .data import superposition_batch  # noqa: F401
from .feed import DeviceActivationPool  # noqa: F401
from .sae import sae_from_tensors  # noqa: F401
from .sharded import ShardedFusedStep, make_shard_sae, shard_range, shard_sae  # noqa: F401
from . import revival  # noqa: F401

__all__ = ["B200JumpReLUSAE", "make_sae", "install", "B200Adam", "FusedStep",
           "reference_param_groups", "superposition_batch", "SaeB200Error", "load_library",
           "sae_from_tensors", "ShardedFusedStep", "shard_sae", "make_shard_sae", "shard_range",
           "DeviceActivationPool"]
