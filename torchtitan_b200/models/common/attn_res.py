"""Block Attention Residuals (parity: reference
``experiments/attention_residual/attn_res.py:48-116``).

Instead of ``h = h + f(h)``, a layer's input is a learned softmax mixture of
the *block outputs* so far: the residual stream is cut into blocks of layers;
``V`` stacks the completed block sums and the current partial sum, keys are
``RMSNorm(V)``, and a per-layer pseudo-query ``w`` (zero-initialised, so the
mixture starts uniform) scores them:

    h = sum_n softmax_n(<w, RMSNorm(V_n)>) V_n

With one block per layer it is Full AttnRes.
"""
from __future__ import annotations

import torch

from .layers import RMSNorm, _local


class _AttnResMix(torch.autograd.Function):
    """``block_attn_res`` as one kernel per direction (``csrc/attn_res.cu``): the blocks are read
    in place, the norm and pseudo-query enter as ``u = g * w``."""

    @staticmethod
    def forward(ctx, w, g, eps, *vs):
        from torchtitan_b200.ops._ext import ext

        vs = [v.contiguous() for v in vs]
        u = (g.float() * w.float().reshape(-1)).contiguous()
        ctx.save_for_backward(w, g, u, *vs)
        ctx.eps = eps
        return ext().attn_res_fwd(vs, u, eps)

    @staticmethod
    def backward(ctx, dout):
        from torchtitan_b200.ops._ext import ext

        w, g, u, *vs = ctx.saved_tensors
        *dvs, du = ext().attn_res_bwd(vs, u, dout.contiguous(), ctx.eps)
        dw = (du * g.float()).reshape(w.shape).to(w.dtype)
        dg = (du * w.float().reshape(-1)).to(g.dtype)
        return (dw, dg, None, *dvs)


def _attn_res_kernel_ok(vs: list[torch.Tensor], query: torch.Tensor, norm) -> bool:
    import os

    if os.environ.get("TTB_ATTNRES_KERNEL", "1") == "0":  # TTB_ATTNRES_KERNEL=0 selects PyTorch
        return False
    w = norm.weight
    return (vs[0].is_cuda and all(v.dtype == torch.bfloat16 and v.shape == vs[0].shape for v in vs)
            and len(vs) <= 17 and type(w).__name__ != "DTensor" and type(query).__name__ != "DTensor")


def block_attn_res(blocks: list[torch.Tensor], partial: torch.Tensor, query: torch.Tensor, norm: RMSNorm):
    """softmax_n(<w, RMSNorm(V_n)>) weighted sum of V = blocks + [partial] (all [B,T,D])."""
    if _attn_res_kernel_ok(blocks + [partial], query, norm):
        return _AttnResMix.apply(query, norm.weight, norm.eps, *blocks, partial)
    V = torch.stack(blocks + [partial], 0)
    Kn = norm(V)
    w = _local(query).reshape(-1).to(Kn.dtype)
    logits = torch.einsum("d,nbtd->nbt", w, Kn).float()
    return torch.einsum("nbt,nbtd->btd", torch.softmax(logits, 0).to(V.dtype), V)


def pack_state(state) -> torch.Tensor:
    """(completed blocks, partial block) -> one ``[n_blocks + 1, B, S, D]`` tensor, the form a
    pipeline stage sends to the next one (its shape is fixed per stage boundary)."""
    blocks, partial = state
    return torch.stack(list(blocks) + [partial])


def unpack_state(x: torch.Tensor):
    """Inverse of ``pack_state``; a plain ``[B, S, D]`` hidden state starts with no blocks."""
    if x.dim() == 3:
        return [], x
    parts = list(x.unbind(0))
    return parts[:-1], parts[-1]


# ---------------------------------------------------------------------------------------
# Pipeline stages that share a rank share completed blocks (behaviour parity: reference
# ``experiments/attention_residual/pipeline_adapter.py``).  With stages placed round-robin
# (stage s on rank s % pp), the rank that runs stage s ran stage s - pp before and still
# holds every block that existed at the end of it, so stage s - 1 sends only the blocks
# completed after that point (plus the partial block).  The held blocks enter stage s as
# detached leaves; a hook on each original block adds the leaf's gradient (summed over
# every later stage of the rank that read it) when the earlier stage runs its backward,
# which the schedule orders after all later stages of the same microbatch.
def completed_blocks(layers_done: int, layers_per_block: int) -> int:
    """Blocks in the stack after layers 0..layers_done-1 (layer i opens one when i % lpb == 0)."""
    return -(-layers_done // layers_per_block)


def setup_stage_cache(parts: list, stage_ids: list[int], fqns: list[list[str]], pp: int,
                      n_microbatches: int, layers_per_block: int) -> None:
    done, counts = 0, []
    for names in fqns:
        ids = [int(n.split(".")[1]) for n in names if n.startswith("layers.")]
        done = max([done] + [i + 1 for i in ids])
        counts.append(completed_blocks(done, layers_per_block))
    shared: dict = {}
    for part, sid in zip(parts, stage_ids):
        part._attnres_pp = {"stage": sid, "pp": pp, "n_stages": len(fqns), "counts": counts,
                            "n_mb": n_microbatches, "cache": shared, "calls": 0, "mb": 0}


def _held(cfg, stage: int) -> int:
    """Blocks this stage's rank holds from its previous stage (0 for a rank's first stage)."""
    prev = stage - cfg["pp"]
    return cfg["counts"][prev] if prev >= 0 else 0


def stage_enter(model, x: torch.Tensor | None = None, state=None):
    """State at the start of a pipeline stage: ``state`` on the first stage, else unpacked from
    the received tensor ``x`` (with the rank's held blocks in front when caching is on)."""
    cfg = getattr(model, "_attnres_pp", None)
    if cfg is not None:
        probe = x if x is not None else state[1]
        if probe.device.type != "meta":  # shape inference runs are not microbatches
            cfg["mb"] = cfg["calls"] % cfg["n_mb"]
            cfg["calls"] += 1
    if state is not None:
        return state
    blocks, partial = unpack_state(x)
    if cfg is None or cfg["stage"] < cfg["pp"]:
        return blocks, partial
    if x.device.type == "meta":  # shape inference: stand-ins for the held blocks
        return [torch.empty_like(partial) for _ in range(_held(cfg, cfg["stage"]))] + blocks, partial
    held = cfg["cache"].get(cfg["mb"], [])
    if len(held) != _held(cfg, cfg["stage"]):
        raise RuntimeError(f"AttnRes stage cache: {len(held)} held blocks, expected {_held(cfg, cfg['stage'])}")
    return list(held) + blocks, partial


def stage_exit(model, state) -> torch.Tensor:
    """Packed state for the next stage: with caching, only the blocks its rank lacks."""
    blocks, partial = state
    cfg = getattr(model, "_attnres_pp", None)
    if cfg is None:
        return pack_state(state)
    s = cfg["stage"]
    held = _held(cfg, s)
    if s + cfg["pp"] < cfg["n_stages"] and partial.device.type != "meta":
        # keep every block for this rank's next stage; bridge gradients back to the originals
        leaves = list(cfg["cache"].get(cfg["mb"], []))[:held]
        for b in blocks[held:]:
            leaf = b.detach().requires_grad_(b.requires_grad)
            if b.requires_grad:
                b.register_hook(lambda g, leaf=leaf: g if leaf.grad is None else g + leaf.grad)
            leaves.append(leaf)
        cfg["cache"][cfg["mb"]] = leaves
    start = _held(cfg, s + 1)
    return pack_state((blocks[start:], partial))
