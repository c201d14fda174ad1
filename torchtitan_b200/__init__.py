"""torchtitan_b200: an LLM pre-training framework built for NVIDIA B200 (sm_100a).

Layers (top to bottom): ``train`` / ``trainer`` (entry point and training loop),
``config`` (Configurable components and the ``--module/--config`` registry),
``components`` (data, loss, optimizers, LR schedule, checkpoint, metrics),
``protocols`` (model / spec / converter / state-dict adapter interfaces),
``models`` (Llama 3 dense, Kimi-Linear hybrid), ``parallel`` (device mesh,
FSDP2, TP/SP, Ulysses and ring CP, EP, PP, activation checkpointing) and
``ops`` (hand-written sm_100a CUDA kernels and their autograd wrappers).
"""

__version__ = "0.1.0"
