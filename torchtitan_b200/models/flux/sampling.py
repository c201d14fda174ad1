"""Latent packing, position ids and rectified-flow sampling for FLUX (behaviour parity:
reference ``models/flux/utils.py:61-180`` and ``inference/sampling.py``).

Rectified flow: ``x_t = (1 - t) x_0 + t * noise``; the model predicts the velocity
``noise - x_0``, and sampling integrates ``dx/dt = v`` from ``t = 1`` (noise) to
``t = 0`` with Euler steps.  The step schedule is uniform in ``t``, optionally
warped towards high noise for long image sequences: ``t' = e^mu / (e^mu + 1/t - 1)``
with ``mu`` linear in the image token count (0.5 at 256 tokens, 1.15 at 4096).
"""
from __future__ import annotations

import math

import torch


def pack_latents(x: torch.Tensor) -> torch.Tensor:
    """[B, C, H, W] -> [B, (H/2)(W/2), C*4]: each token is a 2x2 latent patch (c, dy, dx)."""
    B, C, H, W = x.shape
    return x.view(B, C, H // 2, 2, W // 2, 2).permute(0, 2, 4, 1, 3, 5).reshape(B, (H // 2) * (W // 2), C * 4)


def unpack_latents(x: torch.Tensor, h: int, w: int) -> torch.Tensor:
    """Inverse of ``pack_latents`` for an ``h x w`` latent."""
    B, L, D = x.shape
    C = D // 4
    return x.view(B, h // 2, w // 2, C, 2, 2).permute(0, 3, 1, 4, 2, 5).reshape(B, C, h, w)


def latent_position_ids(B: int, h: int, w: int, device=None) -> torch.Tensor:
    """[B, (h/2)(w/2), 3] ids (0, row, col) of the packed latent tokens."""
    r = torch.arange(h // 2, device=device)
    c = torch.arange(w // 2, device=device)
    ids = torch.stack([torch.zeros(h // 2, w // 2, dtype=torch.long, device=device),
                       r[:, None].expand(-1, w // 2), c[None, :].expand(h // 2, -1)], -1)
    return ids.reshape(1, -1, 3).expand(B, -1, -1)


def text_position_ids(B: int, L: int, device=None) -> torch.Tensor:
    return torch.zeros(B, L, 3, dtype=torch.long, device=device)


def time_shift(mu: float, t: torch.Tensor) -> torch.Tensor:
    return math.exp(mu) / (math.exp(mu) + (1.0 / t - 1.0))


def get_schedule(num_steps: int, image_seq_len: int, base_shift: float = 0.5, max_shift: float = 1.15,
                 shift: bool = True) -> list[float]:
    t = torch.linspace(1.0, 0.0, num_steps + 1, dtype=torch.float64)
    if shift:
        mu = base_shift + (max_shift - base_shift) * (image_seq_len - 256) / (4096 - 256)
        inner = time_shift(mu, t[1:-1])
        t = torch.cat([t[:1], inner, t[-1:]])
    return t.tolist()


@torch.no_grad()
def denoise(model, img: torch.Tensor, img_ids: torch.Tensor, txt: torch.Tensor, txt_ids: torch.Tensor,
            vec: torch.Tensor, timesteps: list[float], cfg_scale: float | None = None,
            neg_txt: torch.Tensor | None = None, neg_vec: torch.Tensor | None = None) -> torch.Tensor:
    """Euler integration of the predicted velocity over ``timesteps`` (descending).
    With ``cfg_scale``, each step also runs the unconditional prompt and uses
    ``v_uncond + cfg_scale * (v_cond - v_uncond)``."""
    B = img.shape[0]
    for t_cur, t_next in zip(timesteps[:-1], timesteps[1:]):
        t = torch.full((B,), t_cur, device=img.device, dtype=torch.float32)
        v = model(img=img, img_ids=img_ids, txt=txt, txt_ids=txt_ids, timesteps=t, y=vec).float()
        if cfg_scale is not None:
            vu = model(img=img, img_ids=img_ids, txt=neg_txt, txt_ids=txt_ids, timesteps=t, y=neg_vec).float()
            v = vu + cfg_scale * (v - vu)
        img = (img.float() + (t_next - t_cur) * v).to(img.dtype)
    return img


@torch.no_grad()
def generate_latents(model, txt: torch.Tensor, vec: torch.Tensor, height: int, width: int, steps: int,
                     cfg_scale: float | None = None, neg_txt=None, neg_vec=None, shift: bool = True,
                     generator: torch.Generator | None = None, z_channels: int = 16) -> torch.Tensor:
    """Noise -> clean latents ``[B, z, height/8, width/8]`` for encoded prompts."""
    B = txt.shape[0]
    h, w = 2 * math.ceil(height / 16), 2 * math.ceil(width / 16)
    dev = txt.device
    noise = torch.randn(B, z_channels, h, w, generator=generator, device=dev, dtype=torch.float32)
    img = pack_latents(noise).to(txt.dtype)
    img_ids = latent_position_ids(B, h, w, dev)
    txt_ids = text_position_ids(B, txt.shape[1], dev)
    ts = get_schedule(steps, img.shape[1], shift=shift)
    out = denoise(model, img, img_ids, txt, txt_ids, vec, ts, cfg_scale, neg_txt, neg_vec)
    return unpack_latents(out.float(), h, w)


def save_image(x: torch.Tensor, path: str) -> None:
    """[3, H, W] in [-1, 1] -> PNG."""
    from PIL import Image

    a = ((x.float().clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).permute(1, 2, 0).cpu().numpy()
    Image.fromarray(a).save(path)
