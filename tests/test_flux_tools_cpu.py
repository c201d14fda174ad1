"""FLUX validation (fixed noise levels, sample images) and the inference entry point (CPU)."""
import os

import torch


def test_flux_validation_and_samples(tmp_path):
    from test_flux_cpu import _small_cfg

    from torchtitan_b200.models.flux.trainer import FluxTrainer
    from torchtitan_b200.models.flux.validate import validate_flux

    cfg = _small_cfg(tmp_path, steps=2)
    cfg.flux_validation_freq = 2
    cfg.flux_validation.steps = 1
    cfg.flux_validation.sample_prompts = ["a cat"]
    cfg.flux_validation.sample_steps = 2
    t = FluxTrainer(cfg)
    t.train()
    v = t.last_validation
    assert set(v) == {"validation/loss"} | {f"validation/loss_t={x:g}" for x in cfg.flux_validation.timesteps}
    assert all(torch.isfinite(torch.tensor(x)) for x in v.values())
    assert os.path.exists(tmp_path / "img" / "step-2" / "0.png")
    assert validate_flux(t, cfg.flux_validation) == v  # fixed noise: the same numbers again
    t.close()


def test_flux_infer_writes_one_image_per_prompt(tmp_path, monkeypatch):
    from torchtitan_b200.models.flux import infer

    prompts = tmp_path / "prompts.txt"
    prompts.write_text("a red house\n\na blue car\n")
    out = tmp_path / "out"
    monkeypatch.chdir(tmp_path)
    written = infer.main([
        "--module", "flux", "--config", "flux_debugmodel", "--dump-folder", str(tmp_path),
        "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
        "--inference.prompts-path", str(prompts), "--inference.save-img-folder", str(out),
        "--inference.img-size", "32", "--inference.denoising-steps", "1", "--inference.cfg-scale", "0"])
    assert sorted(os.path.basename(p) for p in written) == ["img_00000.png", "img_00001.png"]
