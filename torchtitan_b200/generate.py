"""Text generation with a trained model (parity: reference
``scripts/generate/test_generate.py:40-330``).

    python -m torchtitan_b200.generate --module llama3 --flavor debugmodel \\
        [--checkpoint <dcp dir>] [--tokenizer <hf tokenizer dir>] --prompt "..." \\
        [--max-new-tokens 32] [--temperature 0] [--top-k 0] [--seed 0]

Decoder models whose layers use the common grouped-query attention or multi-head latent
attention decode with a KV cache (the prompt once, then one token per step; the flash kernel's bottom-right
causal alignment lets one new query attend to every cached key); other models re-run
over the growing sequence.  With ``--temperature 0`` decoding is greedy.

Launched with torchrun on N ranks, the model runs tensor-parallel over all of them (heads
and MLP columns sharded, logits gathered); every rank decodes the same tokens.  Without ``--tokenizer`` the prompt is a
space-separated list of token ids.
"""
from __future__ import annotations

import argparse
import importlib

import torch


@torch.no_grad()
def _sample(logits, temperature, top_k, generator):
    if temperature <= 0:
        return logits.argmax(-1)
    logits = logits / temperature
    if top_k > 0:
        kth = logits.topk(top_k, -1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    return torch.multinomial(torch.softmax(logits, -1), 1, generator=generator)[:, 0]


def _cache_layers(model) -> list | None:
    """The attention modules to cache, or None when the model cannot decode incrementally."""
    from torchtitan_b200.models.common.attention import GQAttention

    layers = getattr(model, "layers", None)
    if layers is None or not hasattr(model, "rope") or getattr(model, "tok_embeddings", None) is None:
        return None
    atts = []
    for blk in layers.values():
        att = getattr(blk, "attention", None)
        if type(att) is not GQAttention and type(att).__name__ != "MLAttention":
            return None
        if att.cp_hook is not None or getattr(att, "mask_type", "causal") != "causal":
            return None
        atts.append(att)
    return atts


def make_tensor_parallel(model):
    """Tensor-parallel inference over every rank of the default process group (dense
    grouped-query-attention and MLA decoders): returns the rank's TP mesh, or None on one rank."""
    import os

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        return None
    if not dist.is_initialized():
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo")
    from torch.distributed.device_mesh import init_device_mesh

    from torchtitan_b200.parallel.tensor_parallel import apply_tp_llama

    dev = "cuda" if torch.cuda.is_available() and dist.get_backend() == "nccl" else "cpu"
    mesh = init_device_mesh(dev, (world,), mesh_dim_names=("tp",))
    apply_tp_llama(model, mesh, loss_parallel=False, sequence_parallel=False)
    return mesh


def generate(model, prompt: torch.Tensor, max_new_tokens: int, temperature: float = 0.0, top_k: int = 0,
             generator: torch.Generator | None = None, eos_id: int | None = None,
             use_cache: bool = True) -> torch.Tensor:
    """prompt: [B, S] token ids -> [B, S + n] (stops early when every row emitted ``eos_id``)."""
    seq = prompt
    done = torch.zeros(prompt.shape[0], dtype=torch.bool, device=prompt.device)
    atts = _cache_layers(model) if use_cache else None
    if atts is not None:
        for a in atts:
            a.kv_cache = {}
    try:
        pos = 0
        for _ in range(max_new_tokens):
            if atts is None:
                logits = model(seq)[:, -1].float()
            else:
                step = seq[:, pos:]
                positions = torch.arange(pos, seq.shape[1], device=seq.device)[None]
                logits = model(step, positions=positions)[:, -1].float()
                pos = seq.shape[1]
            nxt = _sample(logits, temperature, top_k, generator)
            if eos_id is not None:
                nxt = torch.where(done, torch.full_like(nxt, eos_id), nxt)
                done |= nxt == eos_id
            seq = torch.cat([seq, nxt[:, None]], 1)
            if eos_id is not None and bool(done.all()):
                break
    finally:
        if atts is not None:
            for a in atts:
                a.kv_cache = None
    return seq


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--module", default="llama3")
    ap.add_argument("--flavor", default="debugmodel")
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--prompt", default="1 2 3")
    ap.add_argument("--max-new-tokens", type=int, default=32)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--top-k", type=int, default=0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    import os

    if a.device == "cuda" and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))  # one GPU per rank
        a.device = f"cuda:{torch.cuda.current_device()}"
    spec = importlib.import_module(f"torchtitan_b200.models.{a.module}").model_registry(a.flavor)
    torch.manual_seed(a.seed)
    model = spec.model.build().to(a.device)
    model.init_weights()
    if a.checkpoint:
        from torchtitan_b200.checkpoint_conversion import _load_dcp

        sd = _load_dcp(a.checkpoint, {k: v.cpu() for k, v in model.state_dict().items()})
        model.load_state_dict(sd, strict=False)
    mesh = make_tensor_parallel(model)
    if a.device.startswith("cuda"):
        model = model.to(torch.bfloat16)
        model.rope.init_weights(torch.device("cuda"))  # RoPE tables stay fp32
    model.eval()
    tok = None
    if a.tokenizer:
        from torchtitan_b200.components.tokenizer import HuggingFaceTokenizer

        tok = HuggingFaceTokenizer(tokenizer_path=a.tokenizer)
        ids = tok.encode(a.prompt)
    else:
        ids = [int(t) for t in a.prompt.split()]
    g = torch.Generator(device=a.device).manual_seed(a.seed)
    out = generate(model, torch.tensor([ids], device=a.device), a.max_new_tokens, a.temperature, a.top_k, g,
                   getattr(tok, "eos_id", None))
    new = out[0, len(ids):].tolist()
    if mesh is None or mesh.get_local_rank() == 0:
        print(tok.decode(new) if tok else " ".join(map(str, new)))


if __name__ == "__main__":
    main()
