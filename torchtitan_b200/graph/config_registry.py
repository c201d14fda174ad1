"""Named graph-trainer configs (``--module graph --config <fn>``).

Parity target: ``experiments/graph_trainer/llama3/config_registry.py`` and
``qwen3/config_registry.py`` (``graph_trainer_<family>_<size>``): the family's own training
config turned into a :class:`GraphTrainer` config, activation checkpointing replaced by the
graph's selective-recompute pass.
"""
from __future__ import annotations

import dataclasses

from torchtitan_b200.config import ActivationCheckpointConfig
from torchtitan_b200.models.deepseek_v3 import config_registry as deepseek_v3_configs
from torchtitan_b200.models.llama3 import config_registry as llama3_configs
from torchtitan_b200.models.qwen3 import config_registry as qwen3_configs

from .trainer import GraphCompileConfig, GraphTrainer


def to_graph_trainer_config(base, passes: list[str] | None = None) -> GraphTrainer.Config:
    d = {f.name: getattr(base, f.name) for f in dataclasses.fields(base)}
    recompute = d["activation_checkpoint"].mode != "none"
    d["activation_checkpoint"] = ActivationCheckpointConfig(mode="none")
    default = GraphCompileConfig().passes
    d["compile"] = GraphCompileConfig(passes=list(passes if passes is not None else
                                                  (["selective_recompute"] if recompute else []) + default))
    return GraphTrainer.Config(**d)


def graph_trainer_llama3_debugmodel() -> GraphTrainer.Config:
    return to_graph_trainer_config(llama3_configs.llama3_debugmodel())


def graph_trainer_llama3_debugmodel_cpu() -> GraphTrainer.Config:
    """The CPU/gloo debug config (fp32, seq 512, lbs 4) on the graph trainer."""
    return to_graph_trainer_config(llama3_configs.llama3_debugmodel_cpu())


def graph_trainer_llama3_8b() -> GraphTrainer.Config:
    c = to_graph_trainer_config(llama3_configs.llama3_8b())
    c.compile.passes.append("cudagraph")
    return c


def graph_trainer_qwen3_debugmodel() -> GraphTrainer.Config:
    return to_graph_trainer_config(qwen3_configs.qwen3_debugmodel())


def graph_trainer_qwen3_8b() -> GraphTrainer.Config:
    return to_graph_trainer_config(qwen3_configs.qwen3_8b())


def graph_trainer_qwen3_debugmodel_moe() -> GraphTrainer.Config:
    """MoE on one node without expert parallelism: routing and the padded expert layout trace
    without host reads (CUDA)."""
    return to_graph_trainer_config(qwen3_configs.qwen3_debugmodel_moe())


def graph_trainer_deepseek_v3_debugmodel() -> GraphTrainer.Config:
    return to_graph_trainer_config(deepseek_v3_configs.deepseek_v3_debugmodel())


def graph_trainer_deepseek_v3_16b() -> GraphTrainer.Config:
    return _data_parallel_only(to_graph_trainer_config(deepseek_v3_configs.deepseek_v3_16b()))


def _data_parallel_only(c: GraphTrainer.Config) -> GraphTrainer.Config:
    """The graph trainer shards over data-parallel ranks only: model-parallel degrees of the
    base config fold into FSDP."""
    p = c.parallelism
    p.tensor_parallel_degree = p.context_parallel_degree = p.pipeline_parallel_degree = 1
    p.expert_parallel_degree = p.expert_tensor_parallel_degree = 1
    return c


def graph_trainer_llama3_debugmodel_flex_attn() -> GraphTrainer.Config:
    """Packed documents (block-causal masks): positions and document ids are graph inputs."""
    return to_graph_trainer_config(llama3_configs.llama3_debugmodel_flex_attn())


def graph_trainer_llama3_70b() -> GraphTrainer.Config:
    return _data_parallel_only(to_graph_trainer_config(llama3_configs.llama3_70b()))


def graph_trainer_llama3_405b() -> GraphTrainer.Config:
    return _data_parallel_only(to_graph_trainer_config(llama3_configs.llama3_405b()))


def graph_trainer_deepseek_v3_671b() -> GraphTrainer.Config:
    return _data_parallel_only(to_graph_trainer_config(deepseek_v3_configs.deepseek_v3_671b()))
