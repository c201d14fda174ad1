"""The FLUX.1 image autoencoder (behaviour parity: reference
``models/flux/model/autoencoder.py``): a KL-regularised convolutional VAE
(Rombach et al. 2022, "High-Resolution Image Synthesis with Latent Diffusion
Models") that maps ``[B, 3, H, W]`` images in [-1, 1] to ``[B, z, H/8, W/8]`` latents.

Module names follow the published ``ae.safetensors`` checkpoint layout
(``encoder.down.<i>.block.<j>.conv1`` ...), so ``load_autoencoder`` reads it as is.
The autoencoder is frozen during FLUX training (it only encodes the training
images); its convolutions are cuDNN library calls.
"""
from __future__ import annotations

import os

import torch
import torch.nn as nn
import torch.nn.functional as F


def _gn(c: int) -> nn.GroupNorm:
    return nn.GroupNorm(32, c, eps=1e-6, affine=True)


class ResnetBlock(nn.Module):
    def __init__(self, cin: int, cout: int):
        super().__init__()
        self.norm1, self.conv1 = _gn(cin), nn.Conv2d(cin, cout, 3, padding=1)
        self.norm2, self.conv2 = _gn(cout), nn.Conv2d(cout, cout, 3, padding=1)
        self.nin_shortcut = nn.Conv2d(cin, cout, 1) if cin != cout else None

    def forward(self, x):
        h = self.conv1(F.silu(self.norm1(x)))
        h = self.conv2(F.silu(self.norm2(h)))
        return (self.nin_shortcut(x) if self.nin_shortcut is not None else x) + h


class AttnBlock(nn.Module):
    """Single-head self-attention over the ``H*W`` positions."""

    def __init__(self, c: int):
        super().__init__()
        self.norm = _gn(c)
        self.q, self.k, self.v = nn.Conv2d(c, c, 1), nn.Conv2d(c, c, 1), nn.Conv2d(c, c, 1)
        self.proj_out = nn.Conv2d(c, c, 1)

    def forward(self, x):
        B, C, H, W = x.shape
        h = self.norm(x)
        q, k, v = (m(h).flatten(2).transpose(1, 2)[:, None] for m in (self.q, self.k, self.v))
        o = F.scaled_dot_product_attention(q, k, v)[:, 0].transpose(1, 2).reshape(B, C, H, W)
        return x + self.proj_out(o)


class Downsample(nn.Module):
    def __init__(self, c: int):
        super().__init__()
        self.conv = nn.Conv2d(c, c, 3, stride=2)

    def forward(self, x):
        return self.conv(F.pad(x, (0, 1, 0, 1)))


class Upsample(nn.Module):
    def __init__(self, c: int):
        super().__init__()
        self.conv = nn.Conv2d(c, c, 3, padding=1)

    def forward(self, x):
        return self.conv(F.interpolate(x, scale_factor=2.0, mode="nearest"))


class _Level(nn.Module):
    pass


class _Mid(nn.Module):
    def __init__(self, c: int):
        super().__init__()
        self.block_1, self.attn_1, self.block_2 = ResnetBlock(c, c), AttnBlock(c), ResnetBlock(c, c)

    def forward(self, x):
        return self.block_2(self.attn_1(self.block_1(x)))


class Encoder(nn.Module):
    def __init__(self, in_ch: int, ch: int, ch_mult: tuple[int, ...], num_res_blocks: int, z_channels: int):
        super().__init__()
        self.conv_in = nn.Conv2d(in_ch, ch, 3, padding=1)
        mult = (1,) + tuple(ch_mult)
        self.down = nn.ModuleList()
        for i in range(len(ch_mult)):
            lvl = _Level()
            cin, cout = ch * mult[i], ch * ch_mult[i]
            lvl.block = nn.ModuleList(ResnetBlock(cin if j == 0 else cout, cout) for j in range(num_res_blocks))
            if i != len(ch_mult) - 1:
                lvl.downsample = Downsample(cout)
            self.down.append(lvl)
        c = ch * ch_mult[-1]
        self.mid = _Mid(c)
        self.norm_out = _gn(c)
        self.conv_out = nn.Conv2d(c, 2 * z_channels, 3, padding=1)

    def forward(self, x):
        h = self.conv_in(x)
        for lvl in self.down:
            for blk in lvl.block:
                h = blk(h)
            if hasattr(lvl, "downsample"):
                h = lvl.downsample(h)
        h = self.mid(h)
        return self.conv_out(F.silu(self.norm_out(h)))


class Decoder(nn.Module):
    def __init__(self, out_ch: int, ch: int, ch_mult: tuple[int, ...], num_res_blocks: int, z_channels: int):
        super().__init__()
        c = ch * ch_mult[-1]
        self.conv_in = nn.Conv2d(z_channels, c, 3, padding=1)
        self.mid = _Mid(c)
        up = []
        for i in reversed(range(len(ch_mult))):
            lvl = _Level()
            cout = ch * ch_mult[i]
            lvl.block = nn.ModuleList(ResnetBlock(c if j == 0 else cout, cout) for j in range(num_res_blocks + 1))
            c = cout
            if i != 0:
                lvl.upsample = Upsample(c)
            up.insert(0, lvl)  # stored low-resolution-last, as in the checkpoint
        self.up = nn.ModuleList(up)
        self.norm_out = _gn(c)
        self.conv_out = nn.Conv2d(c, out_ch, 3, padding=1)

    def forward(self, z):
        h = self.mid(self.conv_in(z))
        for lvl in reversed(self.up):
            for blk in lvl.block:
                h = blk(h)
            if hasattr(lvl, "upsample"):
                h = lvl.upsample(h)
        return self.conv_out(F.silu(self.norm_out(h)))


class AutoEncoder(nn.Module):
    def __init__(self, *, in_channels: int = 3, out_ch: int = 3, ch: int = 128, ch_mult=(1, 2, 4, 4),
                 num_res_blocks: int = 2, z_channels: int = 16, scale_factor: float = 0.3611,
                 shift_factor: float = 0.1159):
        super().__init__()
        self.encoder = Encoder(in_channels, ch, tuple(ch_mult), num_res_blocks, z_channels)
        self.decoder = Decoder(out_ch, ch, tuple(ch_mult), num_res_blocks, z_channels)
        self.scale_factor, self.shift_factor = scale_factor, shift_factor

    def encode(self, x: torch.Tensor, sample: bool = False, generator: torch.Generator | None = None) -> torch.Tensor:
        mean, logvar = self.encoder(x).chunk(2, dim=1)
        z = mean
        if sample:
            eps = torch.randn(mean.shape, generator=generator, device=mean.device, dtype=mean.dtype)
            z = mean + torch.exp(0.5 * logvar.clamp(-30.0, 20.0)) * eps
        return self.scale_factor * (z - self.shift_factor)

    def decode(self, z: torch.Tensor) -> torch.Tensor:
        return self.decoder(z / self.scale_factor + self.shift_factor)


def build_autoencoder(args, path: str | None = None, device: torch.device | str = "cpu",
                      dtype: torch.dtype = torch.bfloat16) -> AutoEncoder:
    """The frozen autoencoder of ``FluxModelArgs``; weights from ``path`` (safetensors)
    when it exists, else random (synthetic runs)."""
    ae = AutoEncoder(ch=args.ae_ch, ch_mult=args.ae_ch_mult, num_res_blocks=args.ae_num_res_blocks,
                     z_channels=args.ae_z_channels, scale_factor=args.ae_scale_factor,
                     shift_factor=args.ae_shift_factor)
    if path and os.path.exists(path):
        from safetensors.torch import load_file

        missing, unexpected = ae.load_state_dict(load_file(path), strict=False)
        if missing or unexpected:
            raise ValueError(f"autoencoder checkpoint mismatch: missing {missing[:4]}, unexpected {unexpected[:4]}")
    ae = ae.to(device=device, dtype=dtype).eval()
    for p in ae.parameters():
        p.requires_grad_(False)
    return ae
