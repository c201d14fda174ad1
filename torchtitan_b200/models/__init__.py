_supported_models = frozenset({"llama3", "kimi_linear", "qwen3", "deepseek_v3", "llama4", "gpt_oss", "attention_residual", "hf_transformers", "qwen3_vl", "flux", "vlm"})
