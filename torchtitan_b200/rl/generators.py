"""Rollout generators for the RL loop: this framework's own decoder (``eager``) and vLLM.

Role parity: ``experiments/rl/actors/eager_generator.py`` (the training model itself samples
with a KV cache) and ``actors/generator.py`` + ``models/vllm_wrapper.py`` (a vLLM engine that
receives the trainer's weights every step).  Both return :class:`~.types.Episode` s whose
``token_log_probs`` are the sampling policy's log-probabilities of the sampled tokens; the
trainer uses them as the "old" policy of the clipped surrogate.

Weight sync: the trainer sends its full (unsharded) native state dict; the eager generator
copies it into its parameters, the vLLM generator converts it to the Hugging Face layout
with the family's state-dict adapter and loads it inside the engine's workers
(``LLM.apply_model`` -> ``model.load_weights``).  The vLLM engine is built from a Hugging Face
directory this module writes (``config.json`` + safetensors + the tokenizer files), so no
download is needed.
"""
from __future__ import annotations

import json
import os
from typing import Any, Callable

import torch

from .types import Episode


def _decode(tokenizer, ids: list[int]) -> str:
    if tokenizer is None:
        return " ".join(str(i) for i in ids)
    return tokenizer.decode(ids)


class EagerGenerator:
    """Samples with this framework's model and KV cache (CPU or one GPU).

    ``model_args`` builds the architecture; ``dtype`` is the compute dtype of the copy."""

    def __init__(self, model_args: Any, device: str = "cpu", dtype: str = "float32", seed: int = 0,
                 tokenizer_path: str | None = None):
        self.device = torch.device(device)
        with torch.device(self.device):
            self.model = model_args.build()
        self.model.init_weights()
        self.model.to(getattr(torch, dtype))
        for p in self.model.parameters():
            p.requires_grad_(False)
        self.model.eval()
        self.gen = torch.Generator(device=self.device).manual_seed(seed)
        self.version = -1
        self.tokenizer = None
        if tokenizer_path:
            from torchtitan_b200.components.tokenizer import HuggingFaceTokenizer

            self.tokenizer = HuggingFaceTokenizer(tokenizer_path=tokenizer_path)

    @torch.no_grad()
    def load_state_dict(self, state: dict[str, torch.Tensor], version: int) -> None:
        params = dict(self.model.named_parameters())
        for k, v in state.items():
            params[k].copy_(v.to(params[k].device, params[k].dtype))
        self.version = version

    @torch.no_grad()
    def generate(self, prompts: list[list[int]], n: int, max_new_tokens: int, temperature: float = 1.0,
                 top_k: int = 0, eos_id: int | None = None, expected_answers: list[str] | None = None,
                 group_ids: list[str] | None = None) -> list[Episode]:
        from torchtitan_b200.generate import generate

        from .grpo import token_logprobs

        out: list[Episode] = []
        for i, prompt in enumerate(prompts):
            rep = torch.tensor([prompt] * n, device=self.device)
            seq = generate(self.model, rep, max_new_tokens, temperature, top_k, self.gen, eos_id)
            L = len(prompt)
            lp = token_logprobs(self.model, seq, L)
            if temperature not in (0.0, 1.0):
                # log-probabilities of the tempered distribution that was sampled
                logits = self.model(seq[:, :-1]).float()[:, L - 1:] / temperature
                lp = torch.log_softmax(logits, -1).gather(-1, seq[:, L:, None]).squeeze(-1)
            for j in range(n):
                ids = seq[j, L:].tolist()
                lps = lp[j].tolist()
                if eos_id is not None and eos_id in ids:
                    cut = ids.index(eos_id) + 1
                    ids, lps = ids[:cut], lps[:cut]
                out.append(Episode(policy_version=self.version, prompt_token_ids=list(prompt),
                                   text=_decode(self.tokenizer, ids), token_ids=ids, token_log_probs=lps,
                                   expected_answer=(expected_answers or [""] * len(prompts))[i],
                                   group_id=(group_ids or [str(k) for k in range(len(prompts))])[i]))
        return out


def hf_config(family: str, a: Any) -> dict:
    """Hugging Face ``config.json`` for a Llama 3 or Qwen 3 (dense) model."""
    base = dict(vocab_size=a.vocab_size, hidden_size=a.dim, num_hidden_layers=a.n_layers,
                num_attention_heads=a.n_heads, num_key_value_heads=a.n_kv_heads or a.n_heads,
                rms_norm_eps=a.norm_eps, max_position_embeddings=a.max_seq_len,
                tie_word_embeddings=bool(getattr(a, "enable_weight_tying", False)), torch_dtype="bfloat16",
                rope_theta=a.rope_theta)
    if family == "llama3":
        from torchtitan_b200.models.common.layers import compute_ffn_hidden_dim

        base.update(architectures=["LlamaForCausalLM"], model_type="llama",
                    intermediate_size=compute_ffn_hidden_dim(a.dim, a.multiple_of, a.ffn_dim_multiplier))
        if a.rope_scaling:
            base["rope_scaling"] = {"rope_type": "llama3", "factor": a.rope_scaling_factor, "low_freq_factor": 1.0,
                                    "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}
    elif family == "qwen3":
        if getattr(a, "moe_enabled", False):
            raise NotImplementedError("vLLM export covers dense Qwen3")
        base.update(architectures=["Qwen3ForCausalLM"], model_type="qwen3", intermediate_size=a.hidden_dim,
                    head_dim=a.head_dim)
    else:
        raise NotImplementedError(f"no Hugging Face config writer for {family}")
    return base


def state_dict_adapter(family: str, model_args: Any):
    """The family's native <-> Hugging Face state-dict adapter."""
    import importlib

    mod = importlib.import_module(f"torchtitan_b200.models.{family}")
    return mod.model_registry(next(iter(getattr(mod, f"{family}_args")))).state_dict_adapter(model_args, None)


def write_hf_dir(path: str, family: str, model_args: Any, adapter: Any, state: dict[str, torch.Tensor],
                 tokenizer_path: str | None = None) -> None:
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config(family, model_args), f, indent=1)
    hf = {k: v.detach().to("cpu", torch.bfloat16).contiguous() for k, v in adapter.to_hf(state).items()}
    save_file(hf, os.path.join(path, "model.safetensors"))
    if tokenizer_path:
        import shutil

        for name in ("tokenizer.json", "tokenizer_config.json", "special_tokens_map.json"):
            src = os.path.join(tokenizer_path, name)
            if os.path.exists(src):
                shutil.copy(src, os.path.join(path, name))


def _load_into(weights: list[tuple[str, torch.Tensor]]) -> Callable:
    def fn(model):
        model.load_weights(iter(weights))
        return True

    return fn


class VLLMGenerator:
    """vLLM engine fed with the trainer's weights (one GPU, bf16)."""

    def __init__(self, family: str, model_args: Any, adapter: Any, state: dict[str, torch.Tensor], workdir: str,
                 tokenizer_path: str | None = None, gpu_memory_utilization: float = 0.3, seed: int = 0,
                 enforce_eager: bool = True):
        # the engine runs in this process (the generator is already its own actor process), so
        # weight pushes through apply_model need no serialisation and no forked CUDA context
        os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
        os.environ.setdefault("VLLM_ALLOW_INSECURE_SERIALIZATION", "1")
        from vllm import LLM

        self.adapter = adapter
        path = os.path.join(workdir, "hf_init")
        write_hf_dir(path, family, model_args, adapter, state, tokenizer_path)
        self.llm = LLM(model=path, tokenizer=path if tokenizer_path else None, skip_tokenizer_init=not tokenizer_path,
                       dtype="bfloat16", gpu_memory_utilization=gpu_memory_utilization, seed=seed,
                       enforce_eager=enforce_eager, max_model_len=min(model_args.max_seq_len, 4096))
        self.version = 0

    def load_state_dict(self, state: dict[str, torch.Tensor], version: int) -> None:
        hf = [(k, v.detach().to("cpu", torch.bfloat16).contiguous()) for k, v in self.adapter.to_hf(state).items()]
        self.llm.apply_model(_load_into(hf))
        self.llm.reset_prefix_cache()
        self.version = version

    def generate(self, prompts: list[list[int]], n: int, max_new_tokens: int, temperature: float = 1.0,
                 top_k: int = 0, eos_id: int | None = None, expected_answers: list[str] | None = None,
                 group_ids: list[str] | None = None) -> list[Episode]:
        from vllm import SamplingParams

        sp = SamplingParams(n=n, temperature=temperature, top_k=top_k if top_k > 0 else -1,
                            max_tokens=max_new_tokens, logprobs=0,
                            stop_token_ids=[eos_id] if eos_id is not None else None, ignore_eos=eos_id is None)
        outs = self.llm.generate([{"prompt_token_ids": p} for p in prompts], sp, use_tqdm=False)
        eps = []
        for i, (p, o) in enumerate(zip(prompts, outs)):
            for c in o.outputs:
                ids = list(c.token_ids)
                lps = [float(d[t].logprob) for t, d in zip(ids, c.logprobs)]
                eps.append(Episode(policy_version=self.version, prompt_token_ids=list(p), text=c.text or "",
                                   token_ids=ids, token_log_probs=lps,
                                   expected_answer=(expected_answers or [""] * len(prompts))[i],
                                   group_id=(group_ids or [str(k) for k in range(len(prompts))])[i]))
        return eps
