"""Fetch a Hugging Face repo's tokenizer / config / safetensors files
(parity: reference ``scripts/download_hf_assets.py``).

    python -m torchtitan_b200.download_hf_assets --repo-id meta-llama/Llama-3.1-8B \\
        --assets tokenizer [safetensors config index] --local-dir ./assets/hf [--hf-token ...]
"""
from __future__ import annotations

import argparse
import os

PATTERNS = {
    "tokenizer": ["tokenizer.json", "tokenizer_config.json", "special_tokens_map.json", "tokenizer.model"],
    "config": ["config.json", "generation_config.json"],
    "index": ["model.safetensors.index.json"],
    "safetensors": ["*.safetensors", "model.safetensors.index.json"],
}


def download(repo_id: str, assets: list[str], local_dir: str, token: str | None = None) -> str:
    from huggingface_hub import snapshot_download

    allow = sorted({p for a in assets for p in PATTERNS[a]})
    out = os.path.join(local_dir, repo_id.split("/")[-1])
    snapshot_download(repo_id=repo_id, allow_patterns=allow, local_dir=out, token=token)
    return out


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--repo-id", required=True)
    ap.add_argument("--assets", nargs="+", default=["tokenizer"], choices=sorted(PATTERNS))
    ap.add_argument("--local-dir", default="assets/hf")
    ap.add_argument("--hf-token", default=os.environ.get("HF_TOKEN"))
    a = ap.parse_args(argv)
    print(download(a.repo_id, a.assets, a.local_dir, a.hf_token))


if __name__ == "__main__":
    main()
