"""The model shapes the benchmark and the parity tests run on (random-init,
written as `.gaje.flat` v2 by the synthetic writer).

Each entry is a keyword set for runtime.write_synthetic; arch_family selects
the header's ArchitectureDescriptor (2 SmolLM: RoPE base 1e5; 3 Qwen2 and
4 Qwen2.5: 1e6), which load_genomic applies over the metadata JSON.
"""
from __future__ import annotations

SMOLLM2_135M = dict(arch_family=2, n_embd=576, n_head=9, n_head_kv=3, n_blocks=30, ffn_dim=1536,
                    vocab_size=49152, eps=1e-5, rope_base=100000.0, qkv_bias=False)
QWEN2_0_5B = dict(arch_family=3, n_embd=896, n_head=14, n_head_kv=2, n_blocks=24, ffn_dim=4864,
                  vocab_size=151936, eps=1e-6, rope_base=1000000.0, qkv_bias=True)
QWEN2_5_1_5B = dict(arch_family=4, n_embd=1536, n_head=12, n_head_kv=2, n_blocks=28, ffn_dim=8960,
                    vocab_size=151936, eps=1e-6, rope_base=1000000.0, qkv_bias=True)

# Small shapes for fast parity tests (same code paths, seconds on the CPU oracle).
TINY = dict(arch_family=3, n_embd=128, n_head=4, n_head_kv=2, n_blocks=2, ffn_dim=256,
            vocab_size=512, eps=1e-6, rope_base=1000000.0, qkv_bias=True)
SMALL = dict(arch_family=2, n_embd=256, n_head=8, n_head_kv=2, n_blocks=4, ffn_dim=768,
             vocab_size=4096, eps=1e-5, rope_base=100000.0, qkv_bias=False)

CONFIGS = {
    "smollm2-135m": SMOLLM2_135M,
    "qwen2-0.5b": QWEN2_0_5B,
    # the exporter's --quant-embed variant: Q8_0 token_embd / lm_head
    "qwen2-0.5b-q8e": dict(QWEN2_0_5B, embd_bit_depth=8),
    "qwen2.5-1.5b": QWEN2_5_1_5B,
    "tiny": TINY,
    "small": SMALL,
}


def q4_body_bytes(c: dict) -> int:
    """Algorithmic Q4_0 bytes of the body per decode step (20 bytes per 32 weights)."""
    d, hd = c["n_embd"], c["n_embd"] // c["n_head"]
    qd, kvd, ff = c["n_head"] * hd, c["n_head_kv"] * hd, c["ffn_dim"]
    per_layer = ((qd + 2 * kvd) * d + d * qd + 2 * ff * d + d * ff) // 32 * 20
    return per_layer * c["n_blocks"]


def step_bytes(c: dict, ctx: int) -> dict:
    """Algorithmic HBM bytes of one batch-1 decode step at cache length ctx
    (Q4 body + norms + bias + lm_head (f32, or Q8_0 bytes) + embedding row +
    KV reads)."""
    d, hd = c["n_embd"], c["n_embd"] // c["n_head"]
    qd, kvd = c["n_head"] * hd, c["n_head_kv"] * hd
    L, V = c["n_blocks"], c["vocab_size"]
    body = q4_body_bytes(c)
    norms = (2 * L + 1) * d * 4
    bias = (qd + 2 * kvd) * 4 * L if c.get("qkv_bias") else 0
    q8 = c.get("embd_bit_depth", 32) == 8
    lm = V * (d // 32) * 34 if q8 else V * d * 4  # Q8_0: 34 bytes per 32 weights
    emb = (d // 32) * 34 if q8 else d * 4
    kv = 2 * L * kvd * 4 * ctx
    return dict(body=body, norms=norms, bias=bias, lm_head=lm, embd=emb, kv=kv,
                total=body + norms + bias + lm + emb + kv)
