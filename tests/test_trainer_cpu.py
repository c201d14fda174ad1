"""End-to-end trainer steps on CPU (single process, gloo world of 1)."""
import os

import pytest
import torch

from torchtitan_b200.config.manager import ConfigManager


@pytest.mark.parametrize("module,config,extra", [
    ("llama3", "llama3_debugmodel_cpu", []),
    ("llama3", "llama3_debugmodel", ["--training.seq-len", "128", "--training.local-batch-size", "2",
                                     "--training.dtype", "float32", "--training.mixed-precision-param", "float32"]),
    ("kimi_linear", "kimi_linear_debugmodel", []),
    ("kimi_linear", "kimi_linear_debugmodel_block_attn_res", []),
])
def test_trainer_steps(module, config, extra, tmp_path):
    from torchtitan_b200.trainer import Trainer

    cfg = ConfigManager().parse_args(["--module", module, "--config", config, "--training.steps", "2",
                                      "--dump-folder", str(tmp_path), *extra])
    t = Trainer(cfg)
    t.train()
    loss = t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"]
    assert torch.isfinite(torch.tensor(loss)) and 4.0 < loss < 12.0
    t.close()


@pytest.mark.parametrize("mode,option", [("full", "op"), ("selective", "op"), ("selective", "2")])
def test_activation_checkpointing_is_exact(mode, option, tmp_path):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    def run(extra):
        t = Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel", "--training.steps", "2", "--training.seq-len",
            "64", "--training.local-batch-size", "2", "--training.dtype", "float32",
            "--training.mixed-precision-param", "float32", "--debug.seed", "0", "--metrics.log-freq", "1",
            "--dump-folder", str(tmp_path), *extra]))
        t.train()
        w = {n: p.detach().clone() for n, p in t.model_parts[0].named_parameters()}
        t.close()
        return w

    ref = run(["--activation-checkpoint.mode", "none"])
    got = run(["--activation-checkpoint.mode", mode, "--activation-checkpoint.selective-ac-option", option])
    for n, v in ref.items():
        k = next(k for k in got if k.replace("_checkpoint_wrapped_module.", "") == n.replace(
            "_checkpoint_wrapped_module.", ""))
        torch.testing.assert_close(got[k], v, rtol=0, atol=0, msg=n)
