import torch

from .configurable import Configurable
from .configs import (
    ActivationCheckpointConfig,
    CommConfig,
    CompileConfig,
    DebugConfig,
    ParallelismConfig,
    TrainingConfig,
)

TORCH_DTYPE_MAP = {
    "float16": torch.float16,
    "float32": torch.float32,
    "bfloat16": torch.bfloat16,
}

__all__ = [
    "Configurable",
    "ActivationCheckpointConfig",
    "CommConfig",
    "CompileConfig",
    "DebugConfig",
    "ParallelismConfig",
    "TrainingConfig",
    "TORCH_DTYPE_MAP",
]
