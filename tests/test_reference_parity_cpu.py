"""Loss-curve parity with the reference trainer on the Llama-3 debug model (CPU, gloo,
world size 2, FSDP2, fp32, seq 512, local batch 4, AdamW lr 8e-4 with a 2-step warmup and
linear decay, 10 steps).

Both trainers run in the same two processes: the reference's own ``Trainer`` (its
``llama3_debugmodel`` config through ``Trainer.Config.build()`` and ``Trainer.train_step``;
reference paths ``torchtitan/models/llama3/config_registry.py:33``, ``torchtitan/trainer.py:716``)
and this framework's ``Trainer``. The reference model's initial weights are loaded into ours
(same FQNs), both consume the same token batches, and the ten losses must agree within 1e-4
relative. The reference is imported from its offline install (``baseline/_ref``) or from the
source tree; the only patch is its device selection, which falls back to "cuda" on a host
without a GPU (``torchtitan/tools/utils.py:35-41``).
"""
import os
import sys
import tempfile

import pytest
import torch

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_REF_CANDIDATES = [os.path.join(HERE, "baseline", "_ref"), "/root/reference"]
_REF = next((p for p in _REF_CANDIDATES if os.path.isdir(os.path.join(p, "torchtitan"))), None)

pytestmark = pytest.mark.skipif(_REF is None, reason="reference trainer not available")

STEPS, SEQ, LBS, VOCAB = 10, 512, 4, 2048


def _batches(rank, n):
    out = []
    for i in range(n):
        g = torch.Generator().manual_seed(1234 + 7919 * rank + 104729 * i)
        t = torch.randint(0, VOCAB, (LBS, SEQ + 1), generator=g)
        out.append((t[:, :-1].contiguous(), t[:, 1:].contiguous()))
    return out


def _reference_on_cpu():
    if _REF not in sys.path:
        sys.path.insert(0, _REF)
    import torchtitan.components.metrics as M
    import torchtitan.distributed.parallel_dims as PD
    import torchtitan.distributed.utils as DU
    import torchtitan.tools.utils as U

    for m in (U, PD, DU, M):
        m.device_type = "cpu"
        if hasattr(m, "device_module"):
            m.device_module = torch.cpu

    class _HostMemory:  # the reference's device-memory monitor queries CUDA only
        device_name, device_capacity, device_capacity_gib = "cpu", 1, 1.0

        def get_peak_stats(self):
            return M.DeviceMemStats(0.0, 0.0, 0.0, 0.0, 0, 0)

        def reset_peak_stats(self):
            pass

    M.build_device_memory_monitor = _HostMemory
    # gloo has no PREMUL_SUM, which FSDP2 uses once its gradient division is switched off:
    # keep FSDP's mean reduction and scale the loss by the world size instead (see _run)
    import torchtitan.models.llama3.parallelize as LP

    LP.disable_fsdp_gradient_division = lambda model: None


def _run(rank, world, out_dir, losses_out):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict, set_model_state_dict

    _reference_on_cpu()
    from torchtitan.components.checkpoint import CheckpointManager
    from torchtitan.components.metrics import MetricsProcessor
    from torchtitan.config import ActivationCheckpointConfig, CompileConfig, TrainingConfig
    from torchtitan.models.llama3 import config_registry as ref_reg

    rcfg = ref_reg.llama3_debugmodel()
    rcfg.hf_assets_path = os.path.join(_REF, "tests", "assets", "tokenizer") \
        if os.path.isdir(os.path.join(_REF, "tests", "assets", "tokenizer")) \
        else os.path.join(_REF, "assets", "tokenizer")
    rcfg.training = TrainingConfig(local_batch_size=LBS, seq_len=SEQ, steps=STEPS, mixed_precision_param="float32")
    rcfg.activation_checkpoint = ActivationCheckpointConfig(mode="none")
    rcfg.compile = CompileConfig(enable=False)
    rcfg.checkpoint = CheckpointManager.Config(enable=False)
    rcfg.validator.enable = False
    rcfg.metrics = MetricsProcessor.Config(log_freq=1, enable_tensorboard=False)
    rcfg.dump_folder = os.path.join(out_dir, "ref")
    sys.path.insert(0, HERE)
    from baseline.reference_arm import synthetic_loader_config

    rcfg.dataloader = synthetic_loader_config(VOCAB)  # never consumed: both trainers get the batches below
    ref_losses = []
    ref = rcfg.build()
    base_loss = ref.loss_fn
    ref.loss_fn = lambda pred, labels: base_loss(pred, labels) * world  # FSDP mean x world = sum
    orig_log = ref.metrics_processor.log
    ref.metrics_processor.log = lambda step, avg, mx, *a, **k: (ref_losses.append(avg / world),
                                                                orig_log(step, avg, mx, *a, **k))
    full = get_model_state_dict(ref.model_parts[0], options=StateDictOptions(full_state_dict=True))
    full = {k: v.clone() for k, v in full.items()}

    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    cfg = ConfigManager().parse_args([
        "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", str(STEPS),
        "--metrics.log-freq", "1", "--dump-folder", os.path.join(out_dir, "ours")])
    cfg.model_spec.model.n_kv_heads = 16  # the reference's stock debug model: one KV head per query head
    ours = Trainer(cfg)
    set_model_state_dict(ours.model_parts[0], full, options=StateDictOptions(full_state_dict=True))
    our_losses = []
    orig = ours.metrics_processor.log
    ours.metrics_processor.log = lambda step, avg, mx, *a, **k: (our_losses.append(avg), orig(step, avg, mx, *a, **k))

    batches = _batches(rank, STEPS)
    it_ref = ref.batch_generator([({"input": x}, y) for x, y in batches])
    it_ours = ours.batch_generator([({"input": x}, y) for x, y in batches])
    for _ in range(STEPS):
        ref.step += 1
        ref.train_step(it_ref)
        ours.step += 1
        ours.train_step(it_ours)
    ref.close()
    ours.close()
    if rank == 0:
        torch.save({"ref": ref_losses, "ours": our_losses}, losses_out)


def _entry(rank, world, port, out_dir, losses_out):
    import torch.distributed as dist

    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    try:
        _run(rank, world, out_dir, losses_out)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_debug_model_losses_match_reference_trainer():
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "losses.pt")
        mp.spawn(_entry, args=(2, port, d, out), nprocs=2, join=True)
        res = torch.load(out)
    ref, ours = res["ref"], res["ours"]
    print("reference:", [round(x, 5) for x in ref], "\nours:     ", [round(x, 5) for x in ours])
    assert len(ref) == len(ours) == STEPS, (ref, ours)
    for i, (a, b) in enumerate(zip(ref, ours)):
        assert abs(a - b) <= 1e-4 * abs(a), (i + 1, a, b, ref, ours)
