"""The training loop (parity: ``torchtitan/trainer.py:57-892``).

``Trainer(config)`` sets the device, brings up process groups and meshes,
seeds, builds tokenizer / dataloader / model (on the meta device), applies
converters and parallelism (PP or SPMD), materialises and initialises
weights, then builds optimizers, LR schedulers, checkpointer, validator and
metrics.  ``train()`` runs ``train_step`` until ``training.steps`` with
checkpointing, validation, profiling and PG-timeout tightening after step 1.

``train_step`` collects the gradient-accumulation microbatches on the host,
counts valid tokens globally, copies each microbatch host->device (pinned,
non-blocking), runs forward/backward with loss = local token-sum / global
valid tokens, clips the global grad norm, steps optimizer and scheduler, and
logs (device-timed, max over ranks) every ``metrics.log_freq`` steps.
"""
from __future__ import annotations

import dataclasses
import json
import os
from collections.abc import Iterable, Iterator
from dataclasses import dataclass, field
from datetime import timedelta
from typing import Annotated, Any

import torch
import torch.distributed as dist
import tyro
from torch.distributed.checkpoint.stateful import Stateful

from torchtitan_b200.components.checkpoint import CheckpointManager
from torchtitan_b200.components.dataloader import BaseDataLoader, DataloaderExhaustedError, SyntheticDataLoader
from torchtitan_b200.components.loss import IGNORE_INDEX
from torchtitan_b200.components.lr_scheduler import LRSchedulersContainer
from torchtitan_b200.components.metrics import MetricsProcessor
from torchtitan_b200.components.optimizer import OptimizersContainer
from torchtitan_b200.components.tokenizer import BaseTokenizer, SyntheticTokenizer
from torchtitan_b200.components.validate import Validator
from torchtitan_b200.config import (
    TORCH_DTYPE_MAP,
    ActivationCheckpointConfig,
    CommConfig,
    CompileConfig,
    Configurable,
    DebugConfig,
    ParallelismConfig,
    TrainingConfig,
)
from torchtitan_b200.parallel import ParallelDims
from torchtitan_b200.parallel.semi_sync import FaultToleranceConfig
from torchtitan_b200.parallel import utils as dist_utils
from torchtitan_b200.protocols import ModelConvertersContainer, ModelSpec
from torchtitan_b200.utils import device as dev_utils
from torchtitan_b200.utils.logging import logger
from torchtitan_b200.utils.profiling import ProfilingConfig, maybe_enable_memory_snapshot, maybe_enable_profiling


class Trainer(Stateful, Configurable):
    @dataclass(kw_only=True, slots=True)
    class Config(Configurable.Config):
        model_spec: Annotated[ModelSpec | None, tyro.conf.Suppress] = None
        hf_assets_path: str = "./assets/tokenizer"
        dump_folder: str = "./outputs"
        profiling: ProfilingConfig = field(default_factory=ProfilingConfig)
        metrics: MetricsProcessor.Config = field(default_factory=MetricsProcessor.Config)
        tokenizer: Any = field(default_factory=SyntheticTokenizer.Config)
        dataloader: Any = field(default_factory=SyntheticDataLoader.Config)
        model_converters: ModelConvertersContainer.Config = field(default_factory=ModelConvertersContainer.Config)
        optimizer: OptimizersContainer.Config = field(default_factory=OptimizersContainer.Config)
        lr_scheduler: LRSchedulersContainer.Config = field(default_factory=LRSchedulersContainer.Config)
        training: TrainingConfig = field(default_factory=TrainingConfig)
        parallelism: ParallelismConfig = field(default_factory=ParallelismConfig)
        checkpoint: CheckpointManager.Config = field(default_factory=CheckpointManager.Config)
        activation_checkpoint: ActivationCheckpointConfig = field(default_factory=ActivationCheckpointConfig)
        compile: CompileConfig = field(default_factory=CompileConfig)
        comm: CommConfig = field(default_factory=CommConfig)
        validator: Validator.Config = field(default_factory=Validator.Config)
        debug: DebugConfig = field(default_factory=DebugConfig)
        fault_tolerance: FaultToleranceConfig = field(default_factory=FaultToleranceConfig)

        def to_dict(self) -> dict[str, Any]:
            d = {}
            for f in dataclasses.fields(self):
                v = getattr(self, f.name)
                if f.name == "model_spec":
                    d[f.name] = None if v is None else {"name": v.name, "flavor": v.flavor}
                elif hasattr(v, "to_dict"):
                    d[f.name] = v.to_dict()
                elif dataclasses.is_dataclass(v):
                    d[f.name] = dataclasses.asdict(v)
                else:
                    d[f.name] = v
            return d

    def __init__(self, config: Config, **kw: Any):
        self.config = c = config
        if c.model_spec is None:
            raise ValueError("Trainer.Config.model_spec must be set (use a config_registry function)")
        spec = c.model_spec
        local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if torch.cuda.is_available():
            self.device = torch.device("cuda", local_rank)
            torch.cuda.set_device(self.device)
        else:
            self.device = torch.device("cpu")

        if c.debug.batch_invariant:
            dist_utils.apply_batch_invariant_env()
        world = dist_utils.init_distributed(c.comm, enable_cpu_backend=c.training.enable_cpu_offload,
                                            base_folder=c.dump_folder)
        if c.parallelism.auto_parallel:
            from torchtitan_b200.parallel.auto_parallel import auto_parallelize_config

            plan = auto_parallelize_config(c, world)
            logger.info(f"auto parallel: {plan.describe()}")
        self.parallel_dims = pd = ParallelDims.from_config(c.parallelism, world)
        ft = c.fault_tolerance
        pd.semi_sync_replicas = bool(ft.enable and ft.semi_sync_method)
        if pd.semi_sync_replicas and not pd.dp_replicate_enabled:
            raise ValueError("semi-synchronous training needs data_parallel_replicate_degree > 1 (the replicas)")
        if c.debug.print_config:
            logger.info(json.dumps(c.to_dict(), indent=2))
        if pd.dp_enabled:
            bm = pd.get_mesh("batch")
            dp_degree, dp_rank = bm.size(), bm.get_local_rank()
        else:
            dp_degree, dp_rank = 1, 0
        self.dp_degree = dp_degree
        self.ft = None
        if ft.enable and not ft.semi_sync_method and ft.lighthouse:
            from torchtitan_b200.parallel.ft import FTManager

            if c.parallelism.data_parallel_comm == "peer":
                raise ValueError("dynamic fault-tolerant replicas work with FSDP2/DDP data parallelism, not the "
                                 "peer-memory runtime")
            c.parallelism.data_parallel_comm = "fsdp2"
            self.ft = FTManager(ft.lighthouse, ft.replica_id, max(ft.group_size, ft.replica_id + 1),
                                min_replica_size=ft.min_replica_size, quorum_timeout_s=ft.quorum_timeout_s,
                                collective_timeout_s=ft.process_group_timeout_ms / 1000, backend=ft.process_group)
            dp_degree, dp_rank = self.ft.data_parallel_info(dp_degree, dp_rank)
            logger.info(f"fault-tolerant replica {ft.replica_id} of up to {self.ft.group_size} "
                        f"(min {ft.min_replica_size}), lighthouse {ft.lighthouse}")
        self.gc_handler = dev_utils.GarbageCollection(gc_freq=c.training.gc_freq, debug=c.training.gc_debug)
        dist_utils.set_determinism(pd, self.device, c.debug, distinct_seed_mesh_dims=["pp"])

        self.tokenizer: BaseTokenizer | None = c.tokenizer.build(tokenizer_path=c.hf_assets_path) if c.tokenizer else None
        margs = spec.model
        margs.update_from_config(trainer_config=c)
        if self.tokenizer is not None and hasattr(margs, "vocab_size") and isinstance(self.tokenizer, SyntheticTokenizer):
            self.tokenizer.vocab_size = margs.vocab_size
        self.dataloader: BaseDataLoader = c.dataloader.build(
            dp_world_size=dp_degree, dp_rank=dp_rank, tokenizer=self.tokenizer, seq_len=c.training.seq_len,
            local_batch_size=c.training.local_batch_size)
        self.model_args = margs
        with torch.device("meta"), dev_utils.set_default_dtype(TORCH_DTYPE_MAP[c.training.dtype]):
            model = margs.build()
        converters = c.model_converters.build(parallel_dims=pd)
        converters.convert(model)
        model.verify_module_protocol()
        has_quant = any(getattr(x, "is_quantization", False) for x in converters.converters)
        self.metrics_processor = c.metrics.build(parallel_dims=pd, dump_folder=c.dump_folder,
                                                 pp_schedule=c.parallelism.pipeline_parallel_schedule,
                                                 config_dict=c.to_dict(), has_quantization=has_quant,
                                                 device=self.device)
        nparams, self.metrics_processor.num_flops_per_token = margs.get_nparams_and_flops(model, c.training.seq_len)
        logger.info(f"model {spec.name} {spec.flavor}: {nparams:,} parameters, "
                    f"{self.metrics_processor.num_flops_per_token:.3e} training FLOPs/token")
        self.loss_fn = spec.build_loss_fn(c.compile, parallel_dims=pd)

        gbs = c.training.global_batch_size
        if gbs < 0:
            gbs = c.training.local_batch_size * dp_degree
        if gbs % (c.training.local_batch_size * dp_degree):
            raise ValueError("global_batch_size must be a multiple of local_batch_size * dp degree")
        self.gradient_accumulation_steps = gbs // (c.training.local_batch_size * dp_degree)
        if c.optimizer.early_step_in_backward and (self.gradient_accumulation_steps > 1 or pd.pp_enabled):
            raise ValueError("optimizer.early_step_in_backward needs one microbatch per step and no PP")

        init_device = "cpu" if c.checkpoint.create_seed_checkpoint else self.device.type
        if pd.pp_enabled:
            if spec.pipelining_fn is None:
                raise RuntimeError(f"{spec.name} does not support pipeline parallel")
            self.pp_schedule, self.model_parts, self.pp_has_first_stage, self.pp_has_last_stage = spec.pipelining_fn(
                model, parallel_dims=pd, training=c.training, model_converters=c.model_converters,
                parallelism=c.parallelism, compile_config=c.compile, ac_config=c.activation_checkpoint,
                dump_folder=c.dump_folder, device=self.device, model_config=margs,
                parallelize_fn=spec.parallelize_fn, loss_fn=self._pp_loss)
            del model
            for m in self.model_parts:
                m.to_empty(device=init_device)
                m.init_weights(buffer_device=None)
                m.train()
        else:
            if not c.checkpoint.create_seed_checkpoint:
                model = spec.parallelize_fn(model, parallel_dims=pd, training=c.training,
                                            model_converters=c.model_converters, parallelism=c.parallelism,
                                            compile_config=c.compile, ac_config=c.activation_checkpoint,
                                            dump_folder=c.dump_folder)
            model.to_empty(device=init_device)
            with torch.no_grad():
                model.init_weights(buffer_device=None)
            from torchtitan_b200.parallel.peer_dp import materialize_data_parallel

            materialize_data_parallel(model)
            model.train()
            if c.compile.enable and "model" in c.compile.components:
                self._maybe_capture_cuda_graphs(model)
            self.model_parts = [model]
            self.pp_has_first_stage = self.pp_has_last_stage = True

        self.optimizers = c.optimizer.build(model_parts=self.model_parts)
        if spec.post_optimizer_build_fn is not None:
            spec.post_optimizer_build_fn(self.optimizers, self.model_parts, pd)
        self.semi_sync = None
        if pd.semi_sync_replicas:
            from torchtitan_b200.parallel.semi_sync import SemiSync

            self.semi_sync = SemiSync(ft, self.model_parts, pd.get_mesh("dp_replicate").get_group())
            logger.info(f"semi-synchronous replicas: {ft.semi_sync_method} every {ft.sync_steps} steps "
                        f"({len(self.semi_sync.fragments)} fragments, {pd.dp_replicate} replicas)")
        self.lr_schedulers = c.lr_scheduler.build(optimizers=self.optimizers, training_steps=c.training.steps)
        self.optimizers.register_step_post_hook(lambda *a, **k: converters.post_optimizer_hook(self.model_parts))
        self.metrics_processor.optimizers = self.optimizers
        self.metrics_processor.model_parts = self.model_parts
        self.step = 0
        self.ntokens_seen = 0
        self.checkpointer = c.checkpoint.build(
            dataloader=self.dataloader, model_parts=self.model_parts, optimizers=self.optimizers,
            lr_schedulers=self.lr_schedulers,
            states={"train_state": self, **({"semi_sync": self.semi_sync} if self.semi_sync is not None else {})},
            sd_adapter=spec.state_dict_adapter(margs, c.hf_assets_path) if spec.state_dict_adapter else None,
            base_folder=c.dump_folder)
        self.train_context = dist_utils.get_train_context(False)
        self.validator = None
        if c.validator.enable:
            self.validator = c.validator.build(dp_world_size=dp_degree, dp_rank=dp_rank, tokenizer=self.tokenizer,
                                               parallel_dims=pd, loss_fn=self.loss_fn,
                                               validation_context=self.train_context,
                                               metrics_processor=self.metrics_processor,
                                               seq_len=c.training.seq_len,
                                               local_batch_size=c.training.local_batch_size, device=self.device)
        if self.validator is not None:
            self.validator.loss_step = self._eval_loss_sum
        if c.debug.nonfinite_check:
            from torchtitan_b200.utils.nonfinite import install_nonfinite_hooks

            for m in self.model_parts:
                install_nonfinite_hooks(m)
        logger.info(f"trainer ready: local batch {c.training.local_batch_size}, global batch {gbs}, grad accum "
                    f"{self.gradient_accumulation_steps}, seq {c.training.seq_len}, steps {c.training.steps}")

    # --------------------------------------------------------------- helpers
    def _maybe_capture_cuda_graphs(self, model: torch.nn.Module) -> None:
        """``compile.enable`` with ``compile.backend=cudagraph``: capture each block's forward
        and backward in CUDA graphs where the layout allows (else log why not)."""
        from torchtitan_b200.parallel.cuda_graphs import apply_cuda_graphs, cuda_graphs_applicable

        c = self.config
        if c.compile.backend != "cudagraph":
            logger.warning(f"compile.backend={c.compile.backend}: only 'cudagraph' is implemented; not compiling")
            return
        why = cuda_graphs_applicable(self.parallel_dims, model)
        if why is not None:
            logger.warning(f"compile.enable: blocks not captured in CUDA graphs ({why})")
            return
        apply_cuda_graphs(model, c.training.local_batch_size, c.training.seq_len,
                          model.tok_embeddings.weight.dtype)

    @staticmethod
    def count_valid(labels: torch.Tensor) -> torch.Tensor:
        """Tokens of a microbatch that count toward the step's loss normalisation."""
        return (labels != IGNORE_INDEX).sum()

    def _loss(self, pred: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        m = self.model_parts[-1]
        if getattr(m, "_tp_loss_parallel", False):
            from torchtitan_b200.parallel.tensor_parallel import vocab_parallel_cross_entropy_sum

            return vocab_parallel_cross_entropy_sum(pred, labels, m._tp_group, IGNORE_INDEX, getattr(m, "_tp_rank", None))
        return self.loss_fn(pred, labels)

    @torch.no_grad()
    def _eval_loss_sum(self, input_dict: dict, labels: torch.Tensor) -> torch.Tensor:
        """Summed validation loss of this rank's share of a batch, through the training layout."""
        inputs, labels, extra_inputs, extra_kwargs = self.post_dataloading_process(input_dict, labels)
        if self.parallel_dims.pp_enabled:
            self._pp_token_norm = 1.0
            comp = getattr(self.model_parts[0], "_fsdp_grad_compensation", 1)
            targets, losses = (labels, []) if self.pp_has_last_stage else (None, None)
            args = (inputs,) if self.pp_has_first_stage else ()
            self.pp_schedule.eval(*args, **extra_kwargs, target=targets, losses=losses)
            if self.pp_has_last_stage:
                return torch.sum(torch.stack(losses)).float().cpu() / comp
            return torch.zeros(())
        pred = self.model_parts[0](inputs, **extra_inputs, **extra_kwargs)
        return self._loss(pred, labels).float().cpu()

    def _pp_loss(self, pred, labels):
        # the schedule backpropagates this value: normalise by the step's global token count
        # here, as the non-PP path does before its backward
        comp = getattr(self.model_parts[0], "_fsdp_grad_compensation", 1)  # see forward_backward_step
        return self._loss(pred, labels) / self._pp_token_norm * comp

    def batch_generator(self, data: Iterable) -> Iterator:
        it = iter(data)
        while True:
            import time as _t

            t0 = _t.perf_counter()
            try:
                inp, labels = next(it)
            except StopIteration as e:
                raise DataloaderExhaustedError() from e
            n = labels.numel()
            self.ntokens_seen += n
            self.metrics_processor.ntokens_since_last_log += n
            self.metrics_processor.data_loading_times.append(_t.perf_counter() - t0)
            yield inp, labels

    def post_dataloading_process(self, input_dict: dict[str, torch.Tensor], labels: torch.Tensor):
        inputs = input_dict["input"]
        extra_inputs = {k: v for k, v in input_dict.items() if k not in ("input", "positions")}
        extra_kwargs: dict[str, Any] = {}
        pos = input_dict.get("positions")
        margs = self.model_args
        if getattr(margs, "mask_type", "causal") == "block_causal" and pos is not None:
            extra_kwargs["positions"] = pos
            extra_kwargs["attention_masks"] = torch.cumsum((pos == 0).int(), dim=1)
        pd = self.parallel_dims
        if pd.cp_enabled:
            from torchtitan_b200.parallel.context_parallel import prepare_context_parallel_input

            inputs, labels, extra_kwargs = prepare_context_parallel_input(
                inputs, labels, extra_kwargs, pd.get_mesh("cp"), self.device,
                self.config.parallelism.context_parallel_load_balancer,
                self.config.parallelism.context_parallel_method)
        # pipeline stages check shapes and strides of what they receive
        return inputs.contiguous(), labels.contiguous(), extra_inputs, extra_kwargs

    def forward_backward_step(self, *, input_dict, labels, global_valid_tokens) -> torch.Tensor:
        inputs, labels, extra_inputs, extra_kwargs = self.post_dataloading_process(input_dict, labels)
        pd = self.parallel_dims
        if pd.pp_enabled:
            self._pp_token_norm = global_valid_tokens
            with self.train_context():
                targets, losses = (labels, []) if self.pp_has_last_stage else (None, None)
                if self.pp_has_first_stage:
                    self.pp_schedule.step(inputs, **extra_kwargs, target=targets, losses=losses)
                else:
                    self.pp_schedule.step(**extra_kwargs, target=targets, losses=losses)
            if self.pp_has_last_stage:
                comp = getattr(self.model_parts[0], "_fsdp_grad_compensation", 1)
                return (torch.sum(torch.stack(losses)) / comp).to(self.device)
            return torch.tensor([-1.0], device=self.device)
        with self.train_context():
            pred = self.model_parts[0](inputs, **extra_inputs, **extra_kwargs)
            loss = self._loss(pred, labels) / global_valid_tokens
            del pred
            comp = getattr(self.model_parts[0], "_fsdp_grad_compensation", 1)
            (loss * comp if comp != 1 else loss).backward()
        return loss

    def apply_gradients(self) -> torch.Tensor:
        """Everything after the backward passes of a step: data-parallel gradient finish,
        global-norm clipping (fused into the optimizer where it supports it), optimizer,
        semi-sync and LR-scheduler steps.  Returns the pre-clip gradient norm."""
        pd = self.parallel_dims
        dp_rt = getattr(self.model_parts[0], "_dp_runtime", None)
        if self.ft is not None:
            # cross-replica average, then every participant votes; a failed step is dropped everywhere
            ok = self.ft.allreduce_gradients(self.model_parts)
            if not self.ft.should_commit(ok):
                logger.warning(f"step {self.step}: a replica failed during the step; dropping it")
                self.optimizers.zero_grad()
                self.step -= 1
                return torch.zeros((), device=self.device)
        max_norm = self.config.training.max_norm
        if self.optimizers.config.early_step_in_backward:
            max_norm = 0.0  # parameters already stepped inside backward: nothing left to clip
        fused_clip = max_norm > 0 and all(getattr(o, "supports_fused_clip", False)
                                          for o in self.optimizers.optimizers)
        if dp_rt is not None:
            # gradients live in the data-parallel runtime's fp32 shards
            dp_rt.finish_backward()
            total = dp_rt.grad_sumsq()
            clip = (total.sqrt(), total)
            fused_clip = max_norm > 0
        else:
            clip = dist_utils.clip_grad_norm_([p for m in self.model_parts for p in m.parameters()], max_norm,
                                              pp_mesh=pd.get_optional_mesh("pp"), ep_enabled=pd.ep_enabled,
                                              defer_scaling=fused_clip)
        if dp_rt is not None and not fused_clip:
            grad_norm = clip[0]
        elif fused_clip:
            grad_norm, total = clip
            for o in self.optimizers.optimizers:
                o.pending_clip = (total, max_norm)
        else:
            grad_norm = clip
        self.checkpointer.maybe_wait_for_staging()
        self.optimizers.step()
        if self.semi_sync is not None:
            self.semi_sync.after_step(self.step)
        self.lr_schedulers.step()
        return grad_norm

    def train_step(self, data_iterator: Iterator) -> torch.Tensor:
        if self.ft is not None:
            q = self.ft.start_quorum(self.step - 1)
            if self.ft.heal(self.model_parts, self.optimizers, self.lr_schedulers):
                logger.info(f"healed from replica {q.source} at step {q.source_step}")
                self.step = q.source_step + 1
        self.optimizers.zero_grad()
        lr = self.lr_schedulers.schedulers[0].get_last_lr()[0]
        pd = self.parallel_dims
        mbs = []
        local_valid = 0
        for _ in range(self.gradient_accumulation_steps):
            inp, labels = next(data_iterator)
            local_valid += int(self.count_valid(labels))
            mbs.append((inp, labels))
        local_valid_t = torch.tensor(float(local_valid), device=self.device)
        if pd.semi_sync_replicas:  # each replica normalises by its own tokens
            global_valid = (dist_utils.dist_sum(local_valid_t, pd.get_mesh("dp_shard")) if pd.dp_shard > 1
                            else local_valid_t)
        else:
            global_valid = dist_utils.dist_sum(local_valid_t, pd.get_mesh("batch")) if pd.dp_enabled else local_valid_t
        losses = []
        dp_rt = getattr(self.model_parts[0], "_dp_runtime", None)
        for i, (inp, labels) in enumerate(mbs):
            if dp_rt is not None:
                dp_rt.begin_microbatch(i, len(mbs))
            inp = {k: (v.to(self.device, non_blocking=True) if torch.is_tensor(v) else v) for k, v in inp.items()}
            labels = labels.to(self.device, non_blocking=True)
            losses.append(self.forward_backward_step(input_dict=inp, labels=labels,
                                                     global_valid_tokens=global_valid).detach())
        grad_norm = self.apply_gradients()
        loss = torch.sum(torch.stack([l.reshape(()) for l in losses]))
        self.last_loss = loss
        wd = getattr(dp_rt, "watchdog", None)
        if wd is not None and wd.poll() is not None:  # host read, no CUDA call
            dp_rt.check()
        if not self.metrics_processor.should_log(self.step):
            return loss
        if dp_rt is not None:
            dp_rt.check()
        if pd.pp_enabled:
            # only the last stage computed a loss: every stage logs the last stage's value
            pp = pd.get_mesh("pp")
            t = loss.detach().reshape(-1)[:1].clone().to(self.device if dist.get_backend() != "gloo" else "cpu")
            dist.broadcast(t, src=dist.get_global_rank(pp.get_group(), pp.size() - 1), group=pp.get_group())
            loss = t.reshape(()).to(loss.device)
        if pd.dp_cp_enabled:
            mesh = pd.get_optional_mesh("loss")
            avg = float(dist_utils.dist_sum(loss, mesh))
            if pd.semi_sync_replicas:
                avg /= pd.dp_replicate
            local_avg = loss * global_valid / max(local_valid, 1)
            mx = float(dist_utils.dist_max(local_avg, mesh))
        else:
            avg = mx = float(loss)
        self.metrics_processor.log(self.step, avg, mx, float(grad_norm), extra_metrics={"lr": lr,
                                   "n_tokens_seen": self.ntokens_seen})
        return loss

    def train(self) -> None:
        c = self.config
        self.checkpointer.load(step=c.checkpoint.load_step)
        logger.info(f"training starts at step {self.step + 1}")
        with maybe_enable_profiling(c.profiling, global_step=self.step, base_folder=c.dump_folder) as prof, \
                maybe_enable_memory_snapshot(c.profiling, global_step=self.step, base_folder=c.dump_folder) as mem:
            it = self.batch_generator(self.dataloader)
            while self.step < c.training.steps:
                self.step += 1
                self.gc_handler.run(self.step)
                try:
                    self.train_step(it)
                except DataloaderExhaustedError:
                    logger.warning("ran out of data; stopping")
                    break
                self.checkpointer.save(self.step, last_step=(self.step == c.training.steps))
                if self.validator is not None and self.validator.should_validate(self.step):
                    self.validator.validate(self.model_parts, self.step)
                if prof is not None:
                    prof.step()
                if mem is not None:
                    mem.step()
                if self.step == 1:
                    dist_utils.set_pg_timeouts(timedelta(seconds=c.comm.train_timeout_seconds), self.parallel_dims)
        logger.info("training completed")

    def state_dict(self) -> dict[str, Any]:
        return {"step": self.step, "ntokens_seen": self.ntokens_seen}

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        self.step = int(sd["step"])
        self.ntokens_seen = int(sd["ntokens_seen"])

    def close(self) -> None:
        if getattr(self, "checkpointer", None) is not None:
            self.checkpointer.close()
        if getattr(self, "metrics_processor", None) is not None:
            self.metrics_processor.close()
