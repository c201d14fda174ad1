"""Text generation with a trained model (parity: reference
``scripts/generate/test_generate.py:40-330``).

    python -m torchtitan_b200.generate --module llama3 --flavor debugmodel \\
        [--checkpoint <dcp dir>] [--tokenizer <hf tokenizer dir>] --prompt "..." \\
        [--max-new-tokens 32] [--temperature 0] [--top-k 0] [--seed 0]

Decoding re-runs the model over the growing sequence (no KV cache); with
``--temperature 0`` it is greedy.  Without ``--tokenizer`` the prompt is a
space-separated list of token ids.
"""
from __future__ import annotations

import argparse
import importlib

import torch


@torch.no_grad()
def generate(model, prompt: torch.Tensor, max_new_tokens: int, temperature: float = 0.0, top_k: int = 0,
             generator: torch.Generator | None = None, eos_id: int | None = None) -> torch.Tensor:
    """prompt: [B, S] token ids -> [B, S + n] (stops early when every row emitted ``eos_id``)."""
    seq = prompt
    done = torch.zeros(prompt.shape[0], dtype=torch.bool, device=prompt.device)
    for _ in range(max_new_tokens):
        logits = model(seq)[:, -1].float()
        if temperature <= 0:
            nxt = logits.argmax(-1)
        else:
            logits = logits / temperature
            if top_k > 0:
                kth = logits.topk(top_k, -1).values[:, -1:]
                logits = logits.masked_fill(logits < kth, float("-inf"))
            nxt = torch.multinomial(torch.softmax(logits, -1), 1, generator=generator)[:, 0]
        if eos_id is not None:
            nxt = torch.where(done, torch.full_like(nxt, eos_id), nxt)
            done |= nxt == eos_id
        seq = torch.cat([seq, nxt[:, None]], 1)
        if eos_id is not None and bool(done.all()):
            break
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
    spec = importlib.import_module(f"torchtitan_b200.models.{a.module}").model_registry(a.flavor)
    torch.manual_seed(a.seed)
    model = spec.model.build().to(a.device)
    model.init_weights()
    if a.checkpoint:
        from torchtitan_b200.checkpoint_conversion import _load_dcp

        sd = _load_dcp(a.checkpoint, {k: v.cpu() for k, v in model.state_dict().items()})
        model.load_state_dict(sd, strict=False)
    if a.device == "cuda":
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
    print(tok.decode(new) if tok else " ".join(map(str, new)))


if __name__ == "__main__":
    main()
