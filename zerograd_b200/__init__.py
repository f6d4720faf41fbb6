"""zerograd_b200: B200-native (sm_100a) population evaluation and factor
replay for zerograd's ES optimizer, behind zerograd's own API.

The public names mirror the reference package's hot-path exports
(``src/zerograd/__init__.py:3-48``); all compute runs in libzgb200.so
(hand-written CUDA for sm_100a) through its C ABI.
"""
from ._candidate import (CandidateContext, perturbed_linear, perturbed_table_lookup, perturbed_tied_logits,
                         perturbed_vector)
from ._distributed import (CalibrationResult, DeviceShard, DistributedZeroGrad, ShardResult, allgather_losses,
                           compute_partition_sizes)
from ._exchange import ExchangedReplay
from ._factors import matrix_factors, scaled_factor, table_factors, vector_noise
from ._fitness import shape_centered_loss, validate_losses
from ._keys import candidate_key, group_key, step_key
from ._manifest import Manifest, ManifestEntry, ParameterLayout, ParameterPath, ParameterTree
from ._block import attention, layer_norm, rms_norm
from ._ops import gelu, quantize_int8_columns
from ._graph import CapturedGeneration
from ._optimizer import StepMetrics, ZeroGrad, ZeroGradState
from ._replay import replay, replay_entry
from ._transforms import adamw, apply_updates, sgd
from . import checkpoint, random
from .checkpoint import load_checkpoint, save_checkpoint

__all__ = [
    "attention", "load_checkpoint", "save_checkpoint", "checkpoint",
    "CandidateContext", "CalibrationResult", "CapturedGeneration", "DeviceShard", "DistributedZeroGrad", "ExchangedReplay",
    "Manifest", "ManifestEntry",
    "ParameterLayout", "ParameterPath", "ParameterTree", "ShardResult", "StepMetrics", "ZeroGrad",
    "ZeroGradState", "adamw", "allgather_losses", "apply_updates", "candidate_key", "compute_partition_sizes",
    "gelu", "quantize_int8_columns", "group_key", "layer_norm", "matrix_factors", "perturbed_linear", "perturbed_table_lookup", "perturbed_tied_logits",
    "perturbed_vector", "random", "replay", "replay_entry", "rms_norm", "scaled_factor", "sgd", "shape_centered_loss",
    "step_key", "table_factors", "validate_losses", "vector_noise",
]
