"""FLUX validation (behaviour parity: reference ``models/flux/validate.py``): the
flow-matching loss of held-out image-caption batches at fixed noise levels, and
optionally sampled images for a few prompts.

Every validation sample is evaluated at the same ``timesteps`` (evenly spaced in
(0, 1) by default) with noise from a fixed seed, so successive validations measure the
same quantity; the loss is summed over all target elements of all data-parallel ranks
and divided by their count.  Captions are never dropped here.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import torch

from .data import FluxDataLoader
from .sampling import latent_position_ids, pack_latents, save_image, text_position_ids


@dataclass(kw_only=True, slots=True)
class FluxValidationConfig:
    steps: int = 4
    """Batches per validation."""
    timesteps: list[float] = field(default_factory=lambda: [0.1, 0.3, 0.5, 0.7, 0.9])
    seed: int = 4321
    dataset: str = "synthetic"
    sample_prompts: list[str] = field(default_factory=list)
    sample_steps: int = 20
    cfg_scale: float = 5.0
    save_img_folder: str = "img"


@torch.no_grad()
def validate_flux(trainer, cfg: FluxValidationConfig) -> dict[str, float]:
    """Returns ``{"validation/loss": ..., "validation/loss_t=<t>": ...}`` (and writes sample
    images under ``dump_folder/<save_img_folder>/step-<N>/`` when prompts are given)."""
    import torch.distributed as dist

    model = trainer.model_parts[0]
    was = model.training
    model.eval()
    dl = FluxDataLoader(FluxDataLoader.Config(dataset=cfg.dataset, img_size=trainer.dataloader.config.img_size,
                                              prompt_dropout_prob=0.0, seed=cfg.seed),
                        dp_world_size=trainer.dataloader.dp_world_size, dp_rank=trainer.dataloader.dp_rank,
                        tokenizer=None, seq_len=trainer.config.training.seq_len,
                        local_batch_size=trainer.config.training.local_batch_size)
    dev = trainer.device
    sums = torch.zeros(len(cfg.timesteps), dtype=torch.float64, device=dev)
    count = torch.zeros((), dtype=torch.float64, device=dev)
    g = torch.Generator(device=dev).manual_seed(cfg.seed + trainer.dataloader.dp_rank)
    it = iter(dl)
    for _ in range(cfg.steps):
        inp, images = next(it)
        txt, vec, x0 = trainer.encode_batch(inp["captions"], images)
        B, C, h, w = x0.shape
        ids, tids = latent_position_ids(B, h, w, dev), text_position_ids(B, txt.shape[1], dev)
        for i, tv in enumerate(cfg.timesteps):
            noise = torch.randn(x0.shape, generator=g, device=dev)
            t = torch.full((B,), tv, device=dev)
            xt = (1 - tv) * x0 + tv * noise
            pred = model(img=pack_latents(xt), img_ids=ids, txt=txt, txt_ids=tids, timesteps=t, y=vec)
            sums[i] += trainer.loss_fn(pred, pack_latents(noise - x0)).double()
        count += x0.numel()
    if dist.is_initialized() and trainer.parallel_dims.dp_enabled:
        group = trainer.parallel_dims.get_mesh("batch").get_group()
        dist.all_reduce(sums, group=group)
        dist.all_reduce(count, group=group)
    per_t = (sums / count).tolist()
    out = {"validation/loss": sum(per_t) / len(per_t)}
    out.update({f"validation/loss_t={t:g}": v for t, v in zip(cfg.timesteps, per_t)})
    if cfg.sample_prompts and (not dist.is_initialized() or dist.get_rank() == 0):
        folder = os.path.join(trainer.config.dump_folder, cfg.save_img_folder, f"step-{trainer.step}")
        os.makedirs(folder, exist_ok=True)
        imgs = trainer.generate(cfg.sample_prompts, size=trainer.dataloader.config.img_size, steps=cfg.sample_steps,
                                cfg_scale=cfg.cfg_scale, seed=cfg.seed)
        for k, im in enumerate(imgs):
            save_image(im, os.path.join(folder, f"{k}.png"))
    model.train(was)
    return out
