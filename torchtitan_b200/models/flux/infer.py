"""FLUX text-to-image inference (behaviour parity: reference
``models/flux/inference/infer.py``): one image per line of a prompts file, written
as PNG files; data-parallel ranks split the prompts.

    torchrun --nproc-per-node N -m torchtitan_b200.models.flux.infer \\
        --module flux --config flux_dev --checkpoint.enable --checkpoint.load-step -1 \\
        --inference.prompts-path prompts.txt --inference.save-img-folder out/

The model weights come from the run's checkpoint (``checkpoint.*`` flags), or stay
random when no checkpoint is found (smoke runs).
"""
from __future__ import annotations

import os
import sys
from dataclasses import dataclass


@dataclass(kw_only=True, slots=True)
class InferenceConfig:
    prompts_path: str = "prompts.txt"
    save_img_folder: str = "inference_results"
    local_batch_size: int = 2
    img_size: int = 256
    denoising_steps: int = 50
    cfg_scale: float = 5.0
    """Classifier-free guidance scale (<= 0 disables guidance)."""
    seed: int = 0


def _split_args(argv: list[str]) -> tuple[list[str], dict[str, str]]:
    rest, inf = [], {}
    i = 0
    while i < len(argv):
        a = argv[i]
        if a.startswith("--inference."):
            key = a[len("--inference."):].replace("-", "_")
            if "=" in key:
                key, val = key.split("=", 1)
            else:
                i += 1
                val = argv[i]
            inf[key] = val
        else:
            rest.append(a)
        i += 1
    return rest, inf


def main(argv: list[str] | None = None) -> list[str]:
    import torch
    import torch.distributed as dist

    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.utils.logging import init_logger, logger

    from .sampling import save_image
    from .trainer import FluxTrainer

    init_logger()
    rest, inf_args = _split_args(list(sys.argv[1:] if argv is None else argv))
    icfg = InferenceConfig()
    for k, v in inf_args.items():
        setattr(icfg, k, type(getattr(icfg, k))(v))
    cfg = ConfigManager().parse_args(rest)
    trainer = FluxTrainer(cfg)
    try:
        if cfg.checkpoint.enable:
            trainer.checkpointer.load(step=cfg.checkpoint.load_step)
        with open(icfg.prompts_path) as f:
            prompts = [line.strip() for line in f if line.strip()]
        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        mine = prompts[rank::world]
        os.makedirs(icfg.save_img_folder, exist_ok=True)
        written = []
        for s in range(0, len(mine), icfg.local_batch_size):
            batch = mine[s:s + icfg.local_batch_size]
            imgs = trainer.generate(batch, size=icfg.img_size, steps=icfg.denoising_steps,
                                    cfg_scale=icfg.cfg_scale if icfg.cfg_scale > 0 else None,
                                    seed=icfg.seed + rank * 100003 + s)
            for k, im in enumerate(imgs):
                idx = rank + (s + k) * world  # position of the prompt in the file
                path = os.path.join(icfg.save_img_folder, f"img_{idx:05d}.png")
                save_image(im, path)
                written.append(path)
        logger.info(f"wrote {len(written)} images to {icfg.save_img_folder}")
        return written
    finally:
        trainer.close()
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
