"""Hugging Face safetensors <-> DCP checkpoint conversion (parity: reference
``scripts/checkpoint_conversion/convert_from_hf.py``, ``convert_to_hf.py``).

    python -m torchtitan_b200.checkpoint_conversion from_hf <hf_dir> <dcp_dir> --module llama3 --flavor 8B
    python -m torchtitan_b200.checkpoint_conversion to_hf <dcp_dir> <hf_dir> --module llama3 --flavor 8B

``from_hf`` reads every ``*.safetensors`` file of ``hf_dir``, maps names and
layouts with the family's state-dict adapter and writes a model-only DCP
checkpoint (keys as the trainer's ``model`` state, loadable through
``checkpoint.initial_load_path``).  ``to_hf`` reads a DCP checkpoint written by
the trainer (full ``step-N`` folder or model-only) and writes one
``model.safetensors`` plus an index, in ``--export-dtype``.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os

import torch
import torch.distributed.checkpoint as dcp


def _spec(module: str, flavor: str):
    return importlib.import_module(f"torchtitan_b200.models.{module}").model_registry(flavor)


def _template(spec) -> dict[str, torch.Tensor]:
    """Model state dict with real (CPU) storage, shapes of the flavor."""
    with torch.device("meta"):
        model = spec.model.build()
    model.to_empty(device="cpu")
    return {k: v for k, v in model.state_dict().items()}


def convert_from_hf(hf_dir: str, out_dir: str, module: str, flavor: str) -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    spec = _spec(module, flavor)
    hf = {}
    for f in sorted(os.listdir(hf_dir)):
        if f.endswith(".safetensors"):
            hf.update(load_file(os.path.join(hf_dir, f)))
    native = spec.state_dict_adapter(spec.model, hf_dir).from_hf(hf)
    template = _template(spec)
    missing = [k for k in template if k not in native and not k.endswith(("tokens_per_expert", "expert_bias"))]
    if missing:
        raise KeyError(f"HF checkpoint lacks {len(missing)} tensors, e.g. {missing[:3]}")
    state = {k: native[k].to(template[k].dtype) if k in native else template[k].zero_() for k in template}
    dcp.save(state, checkpoint_id=out_dir, no_dist=True)
    return state


def _load_dcp(dcp_dir: str, template: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    from torch.distributed.checkpoint import FileSystemReader

    keys = set(FileSystemReader(dcp_dir).read_metadata().state_dict_metadata)
    prefixed = any(k.startswith("model.") for k in keys) and not any(k in keys for k in template)
    state = {("model." + k if prefixed else k): v for k, v in template.items() if ("model." + k if prefixed else k) in keys}
    dcp.load(state, checkpoint_id=dcp_dir, no_dist=True)
    return {(k[len("model."):] if prefixed else k): v for k, v in state.items()}


def convert_to_hf(dcp_dir: str, hf_dir: str, module: str, flavor: str, export_dtype: str = "bfloat16") -> dict:
    from safetensors.torch import save_file

    spec = _spec(module, flavor)
    native = _load_dcp(dcp_dir, _template(spec))
    dt = getattr(torch, export_dtype)
    hf = spec.state_dict_adapter(spec.model, None).to_hf(native)
    hf = {k: v.to(dt).contiguous() if v.is_floating_point() else v.contiguous() for k, v in hf.items()}
    os.makedirs(hf_dir, exist_ok=True)
    save_file(hf, os.path.join(hf_dir, "model.safetensors"))
    with open(os.path.join(hf_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": sum(v.numel() * v.element_size() for v in hf.values())},
                   "weight_map": {k: "model.safetensors" for k in hf}}, f, indent=1)
    return hf


def main(argv: list[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("direction", choices=["from_hf", "to_hf"])
    ap.add_argument("src")
    ap.add_argument("dst")
    ap.add_argument("--module", default="llama3")
    ap.add_argument("--flavor", default="8B")
    ap.add_argument("--export-dtype", default="bfloat16")
    a = ap.parse_args(argv)
    if a.direction == "from_hf":
        convert_from_hf(a.src, a.dst, a.module, a.flavor)
    else:
        convert_to_hf(a.src, a.dst, a.module, a.flavor, a.export_dtype)


if __name__ == "__main__":
    main()
