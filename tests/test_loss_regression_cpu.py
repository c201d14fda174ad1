"""Numerics regression: 20 steps of the Llama-3 debug model on CPU (fp32, fixed seed,
deterministic mode) reproduce the committed loss curve (parity: the reference's committed
``tests/assets/losses/llama3_cuda.txt`` check).  A change that moves a loss by more than
1e-4 relative (model, init, optimizer, LR schedule, data order) fails here."""
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _committed() -> list[float]:
    with open(os.path.join(HERE, "assets", "losses", "llama3_debug_cpu.txt")) as f:
        return [float(line.split()[1]) for line in f if line.strip() and not line.startswith("#")]


def test_llama3_debug_loss_curve_matches_committed(tmp_path, monkeypatch):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    monkeypatch.setenv("LOCAL_RANK", "0")
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        cfg = ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "20",
            "--training.seq_len", "128", "--training.local_batch_size", "2", "--checkpoint.no-enable",
            "--validator.no-enable", "--debug.seed", "42", "--debug.deterministic",
            "--dump-folder", str(tmp_path)])
        t = Trainer(cfg)
        it = t.batch_generator(t.dataloader)
        got = []
        while t.step < 20:
            t.step += 1
            got.append(float(t.train_step(it)))
        t.close()
    finally:
        torch.set_num_threads(threads)
    want = _committed()
    assert len(want) == 20
    torch.testing.assert_close(torch.tensor(got), torch.tensor(want), rtol=1e-4, atol=0)
