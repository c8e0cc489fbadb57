"""Random-initialised Qwen3 checkpoints for tests and benchmarks (no network, no real weights).

The real Qwen3-4B checkpoint is not available; BASELINE config c5 specifies a random-init model of
the same architecture (std 0.02, seeded). ``random_qwen3`` builds one with Transformers' own
``Qwen3ForCausalLM`` initialisation and ``save_pretrained`` so that ``Engine(model_path)`` loads it
the way the reference loads a checkpoint (engine/engine.py:124-127).
"""

from __future__ import annotations

import torch

QWEN3_4B = dict(layers=36, hidden=2560, intermediate=9728, vocab=151936)


def qwen3_config(layers: int, hidden: int, intermediate: int, vocab: int, max_pos: int = 262144):
    from transformers import Qwen3Config
    return Qwen3Config(
        hidden_size=hidden, intermediate_size=intermediate, num_hidden_layers=layers,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, vocab_size=vocab,
        max_position_embeddings=max_pos, rope_theta=5e6, rms_norm_eps=1e-6,
        tie_word_embeddings=True, initializer_range=0.02, hidden_act="silu")


def random_model(layers: int, hidden: int, intermediate: int, vocab: int, seed: int = 0,
                 device: str = "cpu"):
    """A Qwen3ForCausalLM with Transformers' initialisation (normal, std 0.02), bf16, sdpa."""
    from transformers import Qwen3ForCausalLM
    cfg = qwen3_config(layers, hidden, intermediate, vocab)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen3ForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


def random_qwen3(path, layers: int, hidden: int, intermediate: int, vocab: int, seed: int = 0):
    """Write a random-init checkpoint to `path` (safetensors + config.json)."""
    model = random_model(layers, hidden, intermediate, vocab, seed)
    model.save_pretrained(str(path))
    return path
