"""Graph-based training: SimpleFSDP, whole-step tracing, FX passes, CUDA-graph replay.

Parity target: ``experiments/graph_trainer/`` of the reference.  ``--module graph --config
graph_trainer_llama3_debugmodel`` selects it from the command line.
"""
from .simple_fsdp import MixedPrecisionPolicy, data_parallel, disable_active_parametrization

__all__ = ["MixedPrecisionPolicy", "data_parallel", "disable_active_parametrization"]
