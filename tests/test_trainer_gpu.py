"""Trainer on one B200: single-replica mixed precision, checkpoint round trip."""
import pytest
import torch

from torchtitan_b200.config.manager import ConfigManager

pytestmark = pytest.mark.gpu


def test_replica_mixed_precision_and_checkpoint(tmp_path):
    from torchtitan_b200.trainer import Trainer

    args = ["--module", "llama3", "--config", "llama3_debugmodel", "--training.steps", "3", "--training.seq-len",
            "256", "--training.local-batch-size", "2", "--dump-folder", str(tmp_path), "--checkpoint.enable",
            "--checkpoint.interval", "3", "--checkpoint.no-last-save-model-only",
            "--activation-checkpoint.mode", "selective"]
    t = Trainer(ConfigManager().parse_args(args))
    w = t.model_parts[0].layers["0"]._checkpoint_wrapped_module.attention.wq.weight
    assert w.dtype == torch.bfloat16 and w._master.dtype == torch.float32
    t.train()
    loss = t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"]
    assert 5.0 < loss < 9.0
    master = w._master.clone()
    t.close()
    t2 = Trainer(ConfigManager().parse_args(args[:5] + ["5"] + args[6:]))
    t2.checkpointer.load()
    w2 = t2.model_parts[0].layers["0"]._checkpoint_wrapped_module.attention.wq.weight
    assert t2.step == 3 and torch.equal(w2._master, master) and torch.equal(w2.data, master.bfloat16())
    t2.close()
