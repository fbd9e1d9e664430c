"""Seeded random-init Llama weights (the benchmark configs use no checkpoints).

Every matrix is drawn from N(0, 0.02) and every RMSNorm weight is 1, in a fixed
order (embedding; per layer q, k, v, o, gate, up, down; lm_head) from one
``torch.Generator``, so the same seed gives the same tensors to the CUDA path,
the CPU checker and the reference run.  Matrices use the nn.Linear layout
``[out_features, in_features]``.
"""
from __future__ import annotations

import torch

LAYER_MATS = ("q", "k", "v", "o", "gate", "up", "down")


def weight_shapes(cfg):
    h, f = cfg["hidden_size"], cfg["intermediate_size"]
    d, hq, hkv = cfg["head_dim"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
    return {"q": (hq * d, h), "k": (hkv * d, h), "v": (hkv * d, h), "o": (h, hq * d),
            "gate": (f, h), "up": (f, h), "down": (h, f)}


def iter_random_llama_weights(cfg, seed=0, dtype=torch.float32, device="cpu", std=0.02,
                              layers=None):
    """Yields (name, tensor) in drawing order, one tensor at a time, so a caller
    that keeps only a shard of each (tensor parallelism) never holds the whole
    model: the 70B shape is 141 GB in bf16.  ``layers`` limits which layer
    indices are made (all by default); skipped layers still consume no random
    numbers, so a partial set is NOT a prefix of the full set's stream beyond
    layer 0."""
    g = torch.Generator(device=device).manual_seed(seed)
    shapes = weight_shapes(cfg)

    def draw(shape):
        t = torch.empty(shape, dtype=torch.float32, device=device)
        t.normal_(0.0, std, generator=g)
        return t.to(dtype)

    yield "embed", draw((cfg["vocab_size"], cfg["hidden_size"]))
    for i in range(cfg["num_hidden_layers"]):
        if layers is not None and i not in layers:
            continue
        for m in LAYER_MATS:
            yield f"layers.{i}.{m}", draw(shapes[m])
        yield f"layers.{i}.input_norm", torch.ones(cfg["hidden_size"], dtype=dtype, device=device)
        yield f"layers.{i}.post_norm", torch.ones(cfg["hidden_size"], dtype=dtype, device=device)
    yield "norm", torch.ones(cfg["hidden_size"], dtype=dtype, device=device)
    yield "lm_head", draw((cfg["vocab_size"], cfg["hidden_size"]))


def random_llama_weights(cfg, seed=0, dtype=torch.float32, device="cpu", std=0.02, layers=None):
    """Returns {name: tensor} (the tensors of iter_random_llama_weights)."""
    return dict(iter_random_llama_weights(cfg, seed, dtype, device, std, layers))
