_supported_models = frozenset({"llama3", "kimi_linear"})
