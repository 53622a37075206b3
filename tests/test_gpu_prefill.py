"""gaje_cuda_prefill against the CPU oracle: a prompt fed in one pass
(whole-prompt tensor-core GEMMs + the causal attention kernel) must leave the
stream as token-by-token forward_core steps do -- the last token's logits
within 1e-3 max relative error and the same argmax, and a cache whose later
decode steps match the oracle's (generate_native_core prefills token by
token, src/nn/llm/forward.rs:215-241).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _oracle_prompt(O, path, prompt):
    ref = O.OracleModel(path)
    ref.set_k_wta_ratio(0.0)
    lr = None
    for i, t in enumerate(prompt):
        lr = ref.forward(int(t), i == 0)
    return ref, lr


def _decode_and_compare(gpu, ref, sid, first, steps):
    tok, worst = first, 0.0
    for _ in range(steps):
        am, lg = gpu.forward_batch([sid], [tok], logits=True)
        lr = ref.forward(tok, False)
        worst = max(worst, _rel(lg[0], lr))
        assert int(am[0]) == int(np.argmax(lr))
        tok = int(am[0])
    return worst


# head_dim 32 (tiny, small: the CUDA-core attention kernel), 64 (SmolLM2 G=3,
# Qwen2 G=7) and 128 (G=6 as Qwen2.5-1.5B, G=2) for the tensor-core kernel
@pytest.mark.parametrize("name,P,rows,over", [
    ("tiny", 37, 64, {}), ("small", 70, 32, {}), ("smollm2-135m", 100, 128, {}), ("qwen2-0.5b", 90, 40, {}),
    ("small", 150, 64, dict(n_embd=768, n_head=6, n_head_kv=1)),
    ("small", 97, 48, dict(n_embd=512, n_head=4, n_head_kv=2))])
def test_prefill_matches_token_by_token(g, O, make_model, name, P, rows, over):
    """rows < P: chunked prefill (later chunks attend to the cached ones)."""
    path = make_model(name, seed=41, **over)
    gpu = g.load_genomic_auto(path, max_ctx=P + 16, max_streams=2, max_prefill=rows)
    gpu.set_k_wta_ratio(0.0)
    rng = np.random.default_rng(P)
    prompt = rng.integers(0, gpu.vocab_size, P)
    am, lg = gpu.prefill(1, prompt, logits=True)
    ref, lr = _oracle_prompt(O, path, prompt)
    assert _rel(lg, lr) <= REL_TOL
    assert am == int(np.argmax(lr))
    assert gpu.stream_len(1) == P
    assert _decode_and_compare(gpu, ref, 1, am, 6) <= REL_TOL


def test_prefill_after_decode_and_between_streams(g, O, make_model):
    """A prompt appended to a stream that already has context, while another
    stream is prefilled independently."""
    path = make_model("smollm2-135m", seed=42)
    gpu = g.load_genomic_auto(path, max_ctx=128, max_streams=3, max_prefill=64)
    gpu.set_k_wta_ratio(0.0)
    rng = np.random.default_rng(9)
    V = gpu.vocab_size
    head = rng.integers(0, V, 5)
    ref0 = O.OracleModel(path)
    ref0.set_k_wta_ratio(0.0)
    for i, t in enumerate(head):
        am = gpu.forward_batch([0], [int(t)])
        lr = ref0.forward(int(t), i == 0)
        assert int(am[0]) == int(np.argmax(lr))
    tail = rng.integers(0, V, 33)
    am0, lg0 = gpu.prefill(0, tail, logits=True)
    for t in tail:
        lr = ref0.forward(int(t), False)
    assert _rel(lg0, lr) <= REL_TOL
    other = rng.integers(0, V, 20)
    am2, lg2 = gpu.prefill(2, other, logits=True)
    ref2, lr2 = _oracle_prompt(O, path, other)
    assert _rel(lg2, lr2) <= REL_TOL
    assert gpu.stream_len(0) == 38 and gpu.stream_len(2) == 20
    assert _decode_and_compare(gpu, ref0, 0, am0, 3) <= REL_TOL
    assert _decode_and_compare(gpu, ref2, 2, am2, 3) <= REL_TOL


def test_prefill_short_prompt_uses_cuda_core_gemms(g, O, make_model):
    """Fewer than 16 rows: the CUDA-core GEMMs inside the prefill pass."""
    path = make_model("qwen2-0.5b", seed=43)
    gpu = g.load_genomic_auto(path, max_ctx=32, max_streams=1, max_prefill=64)
    gpu.set_k_wta_ratio(0.0)
    prompt = np.random.default_rng(1).integers(0, gpu.vocab_size, 9)
    am, lg = gpu.prefill(0, prompt, logits=True)
    ref, lr = _oracle_prompt(O, path, prompt)
    assert _rel(lg, lr) <= REL_TOL and am == int(np.argmax(lr))


def test_prefill_errors(g, make_model):
    path = make_model("tiny", seed=44)
    m = g.load_genomic_auto(path, max_ctx=16, max_streams=1)
    with pytest.raises(ValueError):
        m.prefill(0, [1, 2, 3])
    m = g.load_genomic_auto(path, max_ctx=16, max_streams=1, max_prefill=8)
    with pytest.raises(ValueError):
        m.prefill(1, [1, 2])
    with pytest.raises(ValueError) as e:
        m.prefill(0, list(range(17)))
    assert e.value.status == 8
    m.prefill(0, list(range(16)))
    assert m.stream_len(0) == 16
