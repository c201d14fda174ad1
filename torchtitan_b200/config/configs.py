"""Shared trainer config sections (CLI: ``--<section>.<field>``).

Field names and defaults mirror the reference's public flags
(``torchtitan/config/configs.py:26-420``) so command lines carry over.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Literal


@dataclass(kw_only=True, slots=True)
class TrainingConfig:
    local_batch_size: int = 8
    """Batch size per data-parallel rank."""
    global_batch_size: int = -1
    """Global batch; -1 means local_batch_size * dp degree (no accumulation)."""
    seq_len: int = 2048
    max_norm: float = 1.0
    """Gradient-norm clip threshold (<=0 disables clipping)."""
    steps: int = 10000
    enable_cpu_offload: bool = False
    dtype: Literal["bfloat16", "float32"] = "float32"
    """Dtype the model is built in (master weights)."""
    mixed_precision_param: Literal["bfloat16", "float32"] = "bfloat16"
    """Compute dtype of parameters under data parallelism."""
    mixed_precision_reduce: Literal["float32", "bfloat16"] = "float32"
    gc_freq: int = 50
    gc_debug: bool = False


@dataclass(kw_only=True, slots=True)
class ParallelismConfig:
    data_parallel_replicate_degree: int = 1
    data_parallel_shard_degree: int = -1
    fsdp_reshard_after_forward: Literal["default", "always", "never"] = "default"
    tensor_parallel_degree: int = 1
    disable_loss_parallel: bool = False
    enable_async_tensor_parallel: bool = False
    enable_sequence_parallel: bool = True
    pipeline_parallel_degree: int = 1
    module_fqns_per_model_part: list[list[str]] | None = None
    pipeline_parallel_first_stage_less_layers: int = 1
    pipeline_parallel_last_stage_less_layers: int = 1
    pipeline_parallel_layers_per_stage: int | None = None
    pipeline_parallel_schedule: str = "1F1B"
    pipeline_parallel_schedule_csv: str | None = ""
    pipeline_parallel_attnres_cache: bool = True
    """Attention-Residual models under round-robin stage placement: send each stage only the
    residual blocks its rank does not hold from its previous stage."""
    pipeline_parallel_microbatch_size: int = 1
    context_parallel_degree: int = 1
    context_parallel_load_balancer: str | None = "headtail"
    context_parallel_rotate_method: Literal["allgather", "alltoall"] = "allgather"
    context_parallel_method: Literal["ring", "ulysses"] = "ring"
    """Ring attention (KV rotation) or Ulysses (sequence<->head all-to-all)."""
    expert_parallel_degree: int = 1
    expert_tensor_parallel_degree: int = 1
    expert_parallel_comm_backend: Literal["standard", "fused"] = "standard"
    """``standard`` = NCCL all-to-all; ``fused`` = peer-memory dispatch/combine kernels."""
    auto_parallel: bool = False
    """Choose the layout (dp_replicate/dp_shard/cp/tp, SP, async TP, reshard, AC mode, gradient
    accumulation) with the cost model of ``parallel/auto_parallel.py``, overriding those fields."""
    data_parallel_comm: Literal["auto", "fsdp2", "peer"] = "auto"
    """Pure data parallelism: ``peer`` = replicated bf16 weights + sharded optimizer with
    reduce-scatter / all-gather kernels over NVLink peer memory; ``fsdp2`` = FSDP2 over
    NCCL; ``auto`` = ``peer`` on one node of CUDA devices, else ``fsdp2``."""
    data_parallel_bucket_mb: int = 256


@dataclass(kw_only=True, slots=True)
class ActivationCheckpointConfig:
    mode: Literal["selective", "full", "memory_budget", "none"] = "selective"
    selective_ac_option: str = "op"
    """``op`` for per-op SAC (every second GEMM output kept), ``op_all_mm`` for per-op SAC that
    keeps every GEMM output, or an integer N to checkpoint every N-th block."""
    per_op_sac_force_recompute_mm_shapes_by_fqns: list[str] = field(
        default_factory=lambda: ["moe.router.gate"]
    )
    early_stop: bool = False
    memory_budget: float = 0.5
    preserve_rng_state: bool = False
    determinism_check: str = "default"
    debug: bool = False


@dataclass(kw_only=True, slots=True)
class CompileConfig:
    """``enable`` with ``backend="cudagraph"`` captures every dense decoder block's forward
    and backward in CUDA graphs (no tracing compiler: the kernels are hand-written);
    ``components`` containing "model" selects it.  Other backends are not implemented."""
    enable: bool = False
    components: list[str] = field(default_factory=lambda: ["model", "loss"])
    backend: str = "cudagraph"


@dataclass(kw_only=True, slots=True)
class CommConfig:
    init_timeout_seconds: int = 300
    train_timeout_seconds: int = 100
    trace_buf_size: int = 20000
    save_traces_folder: str = "comm_traces"
    save_traces_file_prefix: str = "rank_"
    mode: Literal["default", "fake_backend", "local_tensor"] = "default"


@dataclass(kw_only=True, slots=True)
class DebugConfig:
    seed: int | None = None
    deterministic: bool = False
    deterministic_warn_only: bool = False
    moe_force_load_balance: bool = False
    detect_anomaly: bool = False
    batch_invariant: bool = False
    print_config: bool = False
    save_config_file: str | None = None
    nonfinite_check: bool = False
    """Forward hooks on every module raise, naming the first module whose output holds a NaN
    or Inf (costs one device-to-host read per module output: debugging only)."""
