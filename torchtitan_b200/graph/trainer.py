"""GraphTrainer: the training step as one traced graph with passes, on SimpleFSDP.

Parity target: ``experiments/graph_trainer/trainer.py`` (``GraphTrainer``) and
``configs.py`` (``GraphTrainerCompileConfig``: ``mode``, ``passes``, ``enable_passes``).
What differs by design: the reference compiles through Dynamo/AOTAutograd and Inductor;
here the step is traced once per input shape with ``make_fx`` (:mod:`.tracer`), edited by
the FX passes of :mod:`.passes`, and run eagerly on the hand-written sm_100a kernels, or
replayed as one CUDA graph (pass name ``cudagraph``).

Everything around the step (data, optimizer, clipping, LR, checkpoints, metrics) is the base
:class:`~torchtitan_b200.trainer.Trainer`'s.  Data parallelism is SimpleFSDP on the
``fsdp`` mesh (``dp_replicate`` > 1 gives HSDP); tensor / context / pipeline / expert
parallelism are not combined with it here (``NotImplementedError``).  Activation
checkpointing is a graph pass (``selective_recompute``), so ``activation_checkpoint.mode``
must be ``none``.
"""
from __future__ import annotations

import copy
import dataclasses
from dataclasses import dataclass, field
from typing import Any, Literal

import torch
import torch.nn as nn

from torchtitan_b200.config import TORCH_DTYPE_MAP
from torchtitan_b200.config.configs import CompileConfig
from torchtitan_b200.trainer import Trainer
from torchtitan_b200.utils.logging import logger

from . import passes as graph_passes
from .simple_fsdp import MixedPrecisionPolicy, data_parallel, disable_active_parametrization
from .tracer import GraphStepRunner, trace_train_step


@dataclass(kw_only=True, slots=True)
class GraphCompileConfig(CompileConfig):
    mode: Literal["aot_fx_trace", "eager"] = "aot_fx_trace"
    """``aot_fx_trace``: trace forward+loss+backward into one FX graph and run it;
    ``eager``: SimpleFSDP without tracing (the debugging baseline)."""
    passes: list[str] = field(default_factory=lambda: ["reshard_after_forward", "transformer_block_bucketing"])
    """Graph passes after the default cleanups (see ``graph.passes.PASSES``) plus ``cudagraph``."""
    enable_passes: bool = True
    """False: run the traced graph as traced (no cleanups, no passes)."""
    bucket_bytes: int = 64 << 20
    """Bucket size of ``auto_bucketing``."""
    precompile_artifact_dir: str = ""
    """Directory of traced-and-passed step graphs: a run stores one per rank and input shape
    (keyed by model, shapes, passes, layout and torch version) and later runs load it instead of
    tracing.  Per rank, because uneven parameter shards bake rank-specific sizes into the graph."""


def parallelize_simple_fsdp(model: nn.Module, *, parallel_dims: Any, training: Any, parallelism: Any,
                            ac_config: Any = None, model_converters: Any = None, **_: Any) -> nn.Module:
    """SimpleFSDP on the data-parallel mesh (parity: ``graph_trainer/llama3/parallelize.py``)."""
    pd = parallel_dims
    if pd.tp_enabled or pd.cp_enabled or pd.pp_enabled or pd.ep_enabled:
        raise NotImplementedError("the graph trainer composes SimpleFSDP data parallelism only "
                                  "(tensor/context/pipeline/expert parallelism use the eager Trainer)")
    if ac_config is not None and ac_config.mode != "none":
        raise ValueError("graph trainer: use the selective_recompute pass instead of activation_checkpoint.mode")
    fp8_types: tuple = ()
    conv = model_converters if model_converters is not None else None
    for c in getattr(conv, "converters", None) or []:
        if getattr(c, "enable_fsdp_float8_all_gather", False) and c.enable_fsdp_float8_all_gather:
            from torchtitan_b200.components.quantization.float8 import Float8Linear

            fp8_types = (Float8Linear,)  # the Float8 converter's linears gather FP8 codes
    mp = MixedPrecisionPolicy(param_dtype=TORCH_DTYPE_MAP[training.mixed_precision_param],
                              reduce_dtype=TORCH_DTYPE_MAP[training.mixed_precision_reduce],
                              fp8_all_gather_modules=fp8_types)
    if pd.dp_replicate > 1 and pd.dp_shard > 1:
        mesh, mode = pd.get_mesh(["dp_replicate", "fsdp"]), "hybrid_shard"
    elif pd.dp_replicate > 1:
        mesh, mode = pd.get_mesh("dp_replicate"), "replicate"
    else:
        mesh, mode = pd.get_mesh("fsdp"), "fully_shard"
    data_parallel(model, mesh, mode, mp)
    init = model.init_weights

    def init_weights(*a, **k):  # initialise the stored shards, not gathered copies
        with disable_active_parametrization():
            return init(*a, **k)

    model.init_weights = init_weights
    logger.info(f"graph trainer: SimpleFSDP {mode} over {mesh.size()} ranks "
                f"(param {mp.param_dtype}, reduce {mp.reduce_dtype})")
    return model


class GraphTrainer(Trainer):
    @dataclass(kw_only=True, slots=True)
    class Config(Trainer.Config):
        compile: GraphCompileConfig = field(default_factory=GraphCompileConfig)

    def __init__(self, config: Config, **kw: Any):
        c = config
        if not isinstance(c.compile, GraphCompileConfig):
            c.compile = GraphCompileConfig(**{f.name: getattr(c.compile, f.name)
                                              for f in dataclasses.fields(CompileConfig)})
        spec = copy.copy(c.model_spec)
        spec.parallelize_fn = parallelize_simple_fsdp
        spec.pipelining_fn = None
        c.model_spec = spec
        c.compile.enable = False  # the base trainer's per-block CUDA graphs do not apply here
        c.parallelism.data_parallel_comm = "fsdp2"  # keep the peer-memory runtime out of the way
        super().__init__(c, **kw)
        self._steps: dict[tuple, GraphStepRunner] = {}
        cc = c.compile
        self._passes = [p for p in cc.passes if p != "cudagraph"]
        # --parallelism.fsdp_reshard_after_forward maps onto the graph pass of the same role
        policy = c.parallelism.fsdp_reshard_after_forward
        if policy == "never":
            self._passes = [p for p in self._passes if p != "reshard_after_forward"]
        elif policy == "always" and "reshard_after_forward" not in self._passes:
            self._passes.insert(0, "reshard_after_forward")
        self._cudagraph = "cudagraph" in cc.passes and self.device.type == "cuda"
        unknown = [p for p in self._passes if p not in graph_passes.PASSES]
        if unknown:
            raise ValueError(f"unknown graph passes {unknown}; available: {sorted(graph_passes.PASSES)} + cudagraph")

    def _artifact_path(self, key: tuple) -> str:
        import hashlib
        import os

        import torch.distributed as dist

        c = self.config
        ident = repr((c.model_spec.name, c.model_spec.flavor, repr(self.model_args), key, self._passes,
                      c.compile.enable_passes, c.compile.bucket_bytes, c.training.mixed_precision_param,
                      c.training.mixed_precision_reduce, c.training.dtype, dist.get_world_size() if
                      dist.is_initialized() else 1, self.device.type, torch.__version__))
        h = hashlib.sha256(ident.encode()).hexdigest()[:16]
        rank = dist.get_rank() if dist.is_initialized() else 0
        return os.path.join(c.compile.precompile_artifact_dir, f"step-{h}-rank{rank}.pt")

    def _trace(self, key: tuple, inputs, labels, norm, extra):
        import os

        cc = self.config.compile
        path = self._artifact_path(key) if cc.precompile_artifact_dir else None
        if path and os.path.exists(path):
            traced = torch.load(path, weights_only=False)
            self.loaded_artifacts = getattr(self, "loaded_artifacts", 0) + 1
            logger.info(f"graph trainer: loaded the traced step from {path}")
            return traced, len(traced.gm.graph.nodes)
        traced = trace_train_step(self.model_parts[0], self._loss, inputs, labels, norm, extra)
        n0 = len(traced.gm.graph.nodes)
        if cc.enable_passes:
            graph_passes.apply_passes(traced, graph_passes.DEFAULT_PASSES + self._passes, bucket_bytes=cc.bucket_bytes)
        if path:
            os.makedirs(os.path.dirname(path), exist_ok=True)
            tmp = path + ".tmp"
            torch.save(traced, tmp)
            os.replace(tmp, path)
        return traced, n0

    def _runner(self, inputs: torch.Tensor, labels: torch.Tensor, norm: torch.Tensor,
                extra: dict[str, torch.Tensor]) -> GraphStepRunner:
        key = (tuple(inputs.shape), inputs.dtype, tuple(labels.shape),
               tuple((n, tuple(v.shape), v.dtype) for n, v in sorted(extra.items())))
        run = self._steps.get(key)
        if run is None:
            model = self.model_parts[0]
            traced, n0 = self._trace(key, inputs, labels, norm, extra)
            executor = None
            if self._cudagraph:
                from .cudagraph import CUDAGraphExecutor

                executor = CUDAGraphExecutor(traced.gm)
            run = GraphStepRunner(model, traced, executor)
            run.copy_static_grads = self.gradient_accumulation_steps > 1
            self._steps[key] = run
            ncoll = sum(1 for n in traced.gm.graph.nodes if n.target in graph_passes.COLLECTIVES)
            logger.info(f"graph trainer: traced step for {key[0]}: {n0} -> {len(traced.gm.graph.nodes)} nodes "
                        f"after passes {self._passes}, {ncoll} collectives"
                        f"{', CUDA graph' if self._cudagraph else ''}")
        return run

    def forward_backward_step(self, *, input_dict, labels, global_valid_tokens) -> torch.Tensor:
        if self.config.compile.mode == "eager":
            return super().forward_backward_step(input_dict=input_dict, labels=labels,
                                                 global_valid_tokens=global_valid_tokens)
        inputs, labels, extra_inputs, extra_kwargs = self.post_dataloading_process(input_dict, labels)
        if extra_inputs:
            raise NotImplementedError("graph trainer: extra model inputs (images) are not traced")
        extra = dict(extra_kwargs)
        if any(not torch.is_tensor(v) for v in extra.values()):
            raise NotImplementedError("graph trainer: non-tensor model keyword arguments are not traced")
        norm = global_valid_tokens.to(torch.float32).reshape(())
        return self._runner(inputs, labels, norm, extra)(inputs, labels, norm, extra)
