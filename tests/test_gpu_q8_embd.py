"""Q8_0 token_embd / lm_head (the exporter's --quant-embed models,
scripts/export_gaje_flat.py:25-32) on the device: the embedding rows are the
reference's q * scale values (blocks.rs:44-48) and the lm_head row dots carry
the Q8_0 arm's |t| < 1e-6 flush (genomic.rs:381-448).  Logits and greedy
tokens against the CPU oracle, which runs the reference's Q8_0 AVX2 kernel,
for every batch-1 engine, the batched step and the prompt pass.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("mega", [pytest.param(1, id="fused"), pytest.param(2, id="mega"),
                                  pytest.param(0, id="phase")])
@pytest.mark.parametrize("name", ["tiny", "small"])
def test_q8_embeddings_single_stream(g, O, make_model, name, mega):
    path = make_model(name, seed=61, embd_bit_depth=8)
    info = g.inspect_flat(path)
    assert info["embd_bit_depth"] == 8 and info["lm_head_bit_depth"] == 8
    gpu = g.load_genomic_auto(path, max_ctx=256, use_megakernel=mega)
    ref = O.OracleModel(path)
    gpu.set_k_wta_ratio(0.0)
    ref.set_k_wta_ratio(0.0)
    rng = np.random.default_rng(8)
    worst = 0.0
    tg = tr = None
    for i, t in enumerate(rng.integers(0, gpu.vocab_size, 10)):
        lg, lr = gpu.forward(int(t), i == 0), ref.forward(int(t), i == 0)
        worst = max(worst, _rel(lg, lr))
    tg, tr = int(np.argmax(lg)), int(np.argmax(lr))
    for _ in range(24):
        assert tg == tr
        lg, lr = gpu.forward(tg), ref.forward(tr)
        worst = max(worst, _rel(lg, lr))
        tg, tr = int(np.argmax(lg)), int(np.argmax(lr))
    assert worst <= REL_TOL, worst


def test_q8_embeddings_batched_and_prefill(g, O, make_model):
    path = make_model("small", seed=62, embd_bit_depth=8)
    gpu = g.load_genomic_auto(path, max_ctx=64, max_streams=3, max_prefill=32)
    gpu.set_k_wta_ratio(0.0)
    refs = [O.OracleModel(path) for _ in range(3)]
    rng = np.random.default_rng(9)
    prompts = [[int(t) for t in rng.integers(0, gpu.vocab_size, n)] for n in (5, 9, 3)]
    toks = []
    for s, (r, p) in enumerate(zip(refs, prompts)):
        r.set_k_wta_ratio(0.0)
        am, lg = gpu.prefill(s, p, logits=True)
        lr = None
        for i, t in enumerate(p):
            lr = r.forward(t, i == 0)
        assert _rel(lg, lr) <= REL_TOL
        assert am == int(np.argmax(lr))
        toks.append(am)
    for _ in range(6):
        am, lg = gpu.forward_batch([0, 1, 2], toks, logits=True)
        for s in range(3):
            lr = refs[s].forward(toks[s])
            assert _rel(lg[s], lr) <= REL_TOL
            assert int(am[s]) == int(np.argmax(lr))
        toks = [int(t) for t in am]
