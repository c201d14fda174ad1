"""FLUX rectified-flow training step (behaviour parity: reference
``models/flux/trainer.py:32-324``).

Per microbatch: encode the images with the frozen autoencoder and the captions with
the frozen T5/CLIP encoders, draw ``t ~ U(0, 1)`` and Gaussian noise per sample,
form ``x_t = (1 - t) x_0 + t * noise``, and regress the model's output on the
velocity ``noise - x_0`` with a summed squared error divided by the number of
target elements in the global batch (every data-parallel rank, every microbatch).
Noise and timesteps come from generators seeded by (seed, step, data-parallel rank,
microbatch), so a resumed run repeats them exactly.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from torchtitan_b200.config import TORCH_DTYPE_MAP
from torchtitan_b200.trainer import Trainer

from torchtitan_b200.utils.logging import logger

from .autoencoder import build_autoencoder
from .encoders import FluxEncoderConfig, FluxTextEncoders
from .sampling import generate_latents, latent_position_ids, pack_latents, text_position_ids
from .validate import FluxValidationConfig, validate_flux


class FluxTrainer(Trainer):
    @dataclass(kw_only=True, slots=True)
    class Config(Trainer.Config):
        encoder: FluxEncoderConfig = field(default_factory=FluxEncoderConfig)
        flux_validation: FluxValidationConfig = field(default_factory=FluxValidationConfig)
        flux_validation_freq: int = 0
        """Validate (fixed-noise-level flow loss, optional samples) every this many steps; 0 = never."""

    def __init__(self, config: Config, **kw: Any):
        super().__init__(config, **kw)
        a = self.model_args
        dt = TORCH_DTYPE_MAP[config.training.mixed_precision_param]
        self._enc_dtype = dt
        self.autoencoder = build_autoencoder(a, config.encoder.autoencoder_path, self.device, dt)
        self.text_encoders = FluxTextEncoders(config.encoder, a.context_in_dim, a.vec_in_dim).to(self.device, dt)
        self._microbatch = 0

    def batch_generator(self, data):
        # count transformer tokens (image patches + text), not pixels
        for inp, labels in super().batch_generator(data):
            lat = labels.shape[-1] // 8
            n = labels.shape[0] * ((lat // 2) ** 2 + self.config.encoder.max_t5_encoding_len)
            self.ntokens_seen += n - labels.numel()
            self.metrics_processor.ntokens_since_last_log += n - labels.numel()
            yield inp, labels

    @torch.no_grad()
    def encode_batch(self, captions: list[str], images: torch.Tensor | None):
        tok = self.text_encoders.tokenize(captions)
        txt, vec = self.text_encoders(tok["t5_tokens"].to(self.device), tok["clip_tokens"].to(self.device))
        lat = None
        if images is not None:
            lat = self.autoencoder.encode(images.to(self.device, self._enc_dtype)).float()
        return txt, vec, lat

    def flow_inputs(self, input_dict, labels) -> dict[str, torch.Tensor]:
        """Encoded, noised and packed model inputs of one microbatch (full sequences) and the
        velocity target: keys img, img_ids, txt, txt_ids, timesteps, y, target."""
        txt, vec, x0 = self.encode_batch(input_dict["captions"], labels)
        B, C, h, w = x0.shape
        g = torch.Generator(device=self.device).manual_seed(
            hash((self.config.debug.seed or 0, self.step, self.dataloader.dp_rank, self._microbatch)) & (2**63 - 1))
        with torch.no_grad():
            noise = torch.randn(x0.shape, generator=g, device=self.device)
            t = torch.rand((B,), generator=g, device=self.device)
            xt = (1 - t.view(-1, 1, 1, 1)) * x0 + t.view(-1, 1, 1, 1) * noise
        return {"img": pack_latents(xt), "img_ids": latent_position_ids(B, h, w, self.device), "txt": txt,
                "txt_ids": text_position_ids(B, txt.shape[1], self.device), "timesteps": t, "y": vec,
                "target": pack_latents(noise - x0)}

    def forward_backward_step(self, *, input_dict, labels, global_valid_tokens) -> torch.Tensor:
        if self.parallel_dims.pp_enabled:
            raise NotImplementedError("FLUX runs without pipeline parallelism")
        model = self.model_parts[0]
        f = self.flow_inputs(input_dict, labels)
        self._microbatch += 1
        # global_valid_tokens counts image elements over the global batch; rescale to latent elements
        norm = global_valid_tokens * (f["target"].numel() / labels.numel())
        pd = self.parallel_dims
        if pd.cp_enabled:  # every rank keeps its contiguous slice of the text and image tokens
            mesh = pd.get_mesh("cp")
            cp, r = mesh.size(), mesh.get_local_rank()
            for k in ("img", "img_ids", "txt", "txt_ids", "target"):
                if f[k].shape[1] % cp:
                    raise ValueError(f"flux context parallel: {k} length {f[k].shape[1]} not divisible by cp={cp}")
                f[k] = f[k].chunk(cp, dim=1)[r]
        target = f.pop("target")
        with self.train_context():
            pred = model(**f)
            loss = self.loss_fn(pred, target) / norm
            del pred
            comp = getattr(model, "_fsdp_grad_compensation", 1)
            (loss * comp if comp != 1 else loss).backward()
        return loss

    def train_step(self, data_iterator):
        self._microbatch = 0
        loss = super().train_step(data_iterator)
        freq = self.config.flux_validation_freq
        if freq > 0 and self.step % freq == 0:
            if self.parallel_dims.cp_enabled:
                logger.warning("flux validation runs full sequences: skipped under context parallelism")
            else:
                self.last_validation = validate_flux(self, self.config.flux_validation)
                logger.info("validation step %d: %s", self.step,
                            ", ".join(f"{k.split('/')[-1]} {v:.4f}" for k, v in self.last_validation.items()))
        return loss

    @torch.no_grad()
    def generate(self, prompts: list[str], size: int = 256, steps: int = 50, cfg_scale: float | None = 5.0,
                 seed: int = 0) -> torch.Tensor:
        """Sample images ``[N, 3, size, size]`` in [-1, 1] for ``prompts``."""
        model = self.model_parts[0]
        was = model.training
        model.eval()
        txt, vec, _ = self.encode_batch(prompts, None)
        neg_txt = neg_vec = None
        if cfg_scale is not None:
            neg_txt, neg_vec, _ = self.encode_batch([""] * len(prompts), None)
        g = torch.Generator(device=self.device).manual_seed(seed)
        lat = generate_latents(model, txt, vec, size, size, steps, cfg_scale, neg_txt, neg_vec,
                               shift=steps > 4, generator=g, z_channels=self.model_args.ae_z_channels)
        img = self.autoencoder.decode(lat.to(self._enc_dtype)).float()
        model.train(was)
        return img
