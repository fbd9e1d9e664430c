"""Model shapes of the benchmark configurations (random-init, no checkpoints)."""

# cfg1: tiny fp32 correctness model
TINY = dict(hidden_size=256, intermediate_size=688, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, head_dim=64, vocab_size=1024, rope_theta=10000.0,
            rms_norm_eps=1e-6)

# cfg3 / cfg4: Llama-3-8B shape
LLAMA3_8B = dict(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                 num_attention_heads=32, num_key_value_heads=8, head_dim=128, vocab_size=128256,
                 rope_theta=500000.0, rms_norm_eps=1e-5)

# cfg5: Llama-3-70B shape
LLAMA3_70B = dict(hidden_size=8192, intermediate_size=28672, num_hidden_layers=80,
                  num_attention_heads=64, num_key_value_heads=8, head_dim=128, vocab_size=128256,
                  rope_theta=500000.0, rms_norm_eps=1e-5)


def param_count(cfg):
    h, f, L, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["vocab_size"]
    d, hq, hkv = cfg["head_dim"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
    per_layer = h * (hq * d) * 2 + h * (hkv * d) * 2 + 3 * h * f + 2 * h
    return L * per_layer + 2 * V * h + h
