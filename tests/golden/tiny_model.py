"""A 2-layer Qwen3-shaped model (hidden 512, 4 query / 1 KV heads of 128,
ffn 768, vocab 1000) with the synthetic Q4_K_M tensor recipe of the engine
(Q6_K attn_v, even-layer ffn_down and token_embd; Q4_K elsewhere; F32 norms),
shared by the golden-vector generator and the tests."""
import q4kb200 as q

SEED = 0x5EED
TINY = dict(layers=2, hidden=512, heads=4, kv_heads=1, head_dim=128, ffn=768, vocab=1000, eps=1e-6, rope_base=1e6)


def tiny_spec(c: dict = TINY) -> dict:
    qd, kvd = c["heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
    spec = {}
    for i in range(c["layers"]):
        p = f"blk.{i}."
        spec[p + "attn_norm.weight"] = (q.F32, c["hidden"], 1)
        spec[p + "attn_q.weight"] = (q.Q4_K, c["hidden"], qd)
        spec[p + "attn_k.weight"] = (q.Q4_K, c["hidden"], kvd)
        spec[p + "attn_v.weight"] = (q.Q6_K, c["hidden"], kvd)
        spec[p + "attn_q_norm.weight"] = (q.F32, c["head_dim"], 1)
        spec[p + "attn_k_norm.weight"] = (q.F32, c["head_dim"], 1)
        spec[p + "attn_output.weight"] = (q.Q4_K, qd, c["hidden"])
        spec[p + "ffn_norm.weight"] = (q.F32, c["hidden"], 1)
        spec[p + "ffn_gate.weight"] = (q.Q4_K, c["hidden"], c["ffn"])
        spec[p + "ffn_up.weight"] = (q.Q4_K, c["hidden"], c["ffn"])
        spec[p + "ffn_down.weight"] = (q.Q6_K if i % 2 == 0 else q.Q4_K, c["ffn"], c["hidden"])
    spec["output_norm.weight"] = (q.F32, c["hidden"], 1)
    spec["token_embd.weight"] = (q.Q6_K, c["hidden"], c["vocab"])
    return spec


def tiny_tensors(c: dict = TINY, seed: int = SEED) -> dict:
    """name -> (type, ne0, ne1, GGUF-layout host data)."""
    return {n: (t, a, b, q.synth_tensor_host(seed, n, t, a, b)) for n, (t, a, b) in tiny_spec(c).items()}


def engine_config(c: dict = TINY, capacity: int = 16):
    cfg = q.EngineConfig()
    cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads = c["layers"], c["hidden"], c["heads"], c["kv_heads"]
    cfg.head_dim, cfg.ffn, cfg.vocab = c["head_dim"], c["ffn"], c["vocab"]
    cfg.eps, cfg.rope_base, cfg.capacity = c["eps"], c["rope_base"], capacity
    cfg.tp_rank, cfg.tp_world, cfg.device = 0, 1, 0
    return cfg
