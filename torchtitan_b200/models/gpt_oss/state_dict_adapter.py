"""GPT-OSS <-> Hugging Face ``GptOssForCausalLM`` (in-memory, dequantized layout) names.

q/k rows *and biases* are permuted between HF's rotate-half layout and the
interleaved RoPE pairs of this framework; expert projections are stored
transposed by HF (``gate_up_proj [E, D, 2I]`` with gate/up interleaved along the
last dim, ``down_proj [E, I, D]``) and as ``[out, in]`` here.
"""
from __future__ import annotations

from torchtitan_b200.models.llama3.state_dict_adapter import Llama3StateDictAdapter

_T = ("moe.experts.mlp1_weight", "moe.experts.mlp2_weight")


class GptOssStateDictAdapter(Llama3StateDictAdapter):
    from_hf_map = {
        "model.embed_tokens.weight": "tok_embeddings.weight",
        "model.layers.{}.self_attn.q_proj.weight": "layers.{}.attention.wq.weight",
        "model.layers.{}.self_attn.q_proj.bias": "layers.{}.attention.wq.bias",
        "model.layers.{}.self_attn.k_proj.weight": "layers.{}.attention.wk.weight",
        "model.layers.{}.self_attn.k_proj.bias": "layers.{}.attention.wk.bias",
        "model.layers.{}.self_attn.v_proj.weight": "layers.{}.attention.wv.weight",
        "model.layers.{}.self_attn.v_proj.bias": "layers.{}.attention.wv.bias",
        "model.layers.{}.self_attn.o_proj.weight": "layers.{}.attention.wo.weight",
        "model.layers.{}.self_attn.o_proj.bias": "layers.{}.attention.wo.bias",
        "model.layers.{}.self_attn.sinks": "layers.{}.attention.sinks",
        "model.layers.{}.mlp.router.weight": "layers.{}.moe.router.gate.weight",
        "model.layers.{}.mlp.router.bias": "layers.{}.moe.router.gate.bias",
        "model.layers.{}.mlp.experts.gate_up_proj": "layers.{}.moe.experts.mlp1_weight",
        "model.layers.{}.mlp.experts.gate_up_proj_bias": "layers.{}.moe.experts.mlp1_bias",
        "model.layers.{}.mlp.experts.down_proj": "layers.{}.moe.experts.mlp2_weight",
        "model.layers.{}.mlp.experts.down_proj_bias": "layers.{}.moe.experts.mlp2_bias",
        "model.layers.{}.input_layernorm.weight": "layers.{}.attention_norm.weight",
        "model.layers.{}.post_attention_layernorm.weight": "layers.{}.ffn_norm.weight",
        "model.norm.weight": "norm.weight",
        "lm_head.weight": "output.weight",
    }

    def _heads(self, key: str) -> int | None:
        a = self.model_args
        if a is None:
            return None
        if key.endswith(("attention.wq.weight", "attention.wq.bias")):
            return a.n_heads
        if key.endswith(("attention.wk.weight", "attention.wk.bias")):
            return a.n_kv_heads
        return None

    def to_hf_tensor(self, native_key, t):
        if native_key.endswith(_T):
            return t.transpose(1, 2).contiguous()
        h = self._heads(native_key)
        if h and t.dim() == 1:
            return self.interleaved_to_halves(t[:, None], h)[:, 0]
        return super().to_hf_tensor(native_key, t)

    def from_hf_tensor(self, native_key, t):
        if native_key.endswith(_T):
            return t.transpose(1, 2).contiguous()
        h = self._heads(native_key)
        if h and t.dim() == 1:
            return self.halves_to_interleaved(t[:, None], h)[:, 0]
        return super().from_hf_tensor(native_key, t)
