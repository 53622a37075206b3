"""Genomic4Bit (16-centroid LUT) tensors on the device against the oracle.

The format: per 32-weight block 16 f32 centroids and 16 bytes of codes, the
code of element 2k in the HIGH nibble of byte k (genomize_4bit_core,
src/compute/quantize/genomize.rs:286-382); GenomicLinear::new expands a table
of 16 (whole matrix) or K/32*16 (per block column) to one per (row, block)
(src/nn/linear/init.rs:109-124); the row dot is genomic_dot_product_4bit
(src/compute/kernels/genomic.rs:149-204), flushed below 1e-6, then the bias.

Bars: dequantised weights bit-exact (w = c[code]); row dots within 1e-5 of
the row's sum of |c x| (the oracle keeps four sequential accumulators, the
GPU a lane per element); whole-model logits within 1e-3 max relative error
and the identical greedy stream.
"""
import numpy as np
import pytest

import flat_numpy

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _tables(rng, N, K, layout):
    nb = K // 32
    n = {"full": N * nb * 16, "column": nb * 16, "shared": 16}[layout]
    cen = np.sort(rng.standard_normal(n).astype(np.float32).reshape(-1, 16), axis=1).reshape(-1) * np.float32(0.05)
    nib = rng.integers(0, 256, N * K // 2).astype(np.uint8)
    return nib, cen


def _expand(nib, cen, N, K):
    """init.rs:109-124 expansion + the code order, as plain numpy."""
    nb = K // 32
    if cen.size == 16:
        full = np.broadcast_to(cen.reshape(1, 1, 16), (N, nb, 16))
    elif cen.size == nb * 16:
        full = np.broadcast_to(cen.reshape(1, nb, 16), (N, nb, 16))
    else:
        full = cen.reshape(N, nb, 16)
    codes = np.stack([nib >> 4, nib & 15], axis=1).reshape(N, nb, 32)
    return np.take_along_axis(full, codes.astype(np.int64), axis=2).reshape(N, K), full


@pytest.mark.parametrize("layout", ["full", "column", "shared"])
@pytest.mark.parametrize("N,K", [(896, 896), (4864, 896), (1536, 8960), (7, 64)])
def test_lut4_dequant_and_gemv(g, O, layout, N, K):
    import torch

    rng = np.random.default_rng(N + K)
    nib, cen = _tables(rng, N, K, layout)
    bias = rng.standard_normal(N).astype(np.float32) * np.float32(0.01)
    m = g.Q4Matrix.from_lut4(nib, cen, N, K, bias=bias)
    w = torch.empty((N, K), dtype=torch.float32, device="cuda")
    m.dequant(w.data_ptr())
    x = rng.standard_normal((3, K)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty((3, N), dtype=torch.float32, device="cuda")
    m.gemv(xd.data_ptr(), y.data_ptr(), 3)
    torch.cuda.synchronize()
    wref, full = _expand(nib, cen, N, K)
    assert np.array_equal(w.cpu().numpy(), wref)
    yg = y.cpu().numpy()
    nb = K // 32
    for i in range(3):
        for r in range(0, N, max(1, N // 97)):  # a spread of rows through the oracle's kernel
            ref = O.lut4_dot(nib[r * nb * 16:(r + 1) * nb * 16], x[i], full[r].reshape(-1), nb) + bias[r]
            scale = float(np.sum(np.abs(wref[r] * x[i]))) + 1e-30
            assert abs(float(yg[i, r]) - ref) <= 1e-5 * scale, (i, r)


@pytest.mark.parametrize("layout", ["full", "column", "shared"])
@pytest.mark.parametrize("name,over", [("tiny", {}), ("small", {}), ("small", {"n_embd": 384, "n_head": 6,
                                                                              "n_head_kv": 3})])
def test_lut4_model_matches_oracle(g, O, tmp_path, layout, name, over):
    """Every body matrix a Genomic4Bit table: 12 prompt tokens then 64 greedy
    steps against the oracle; the model runs on the kernel-per-phase engine."""
    cfg = dict(g.configs.CONFIGS[name])
    cfg.update(over)
    path = str(tmp_path / f"lut4_{name}_{layout}.flat")
    flat_numpy.write_synthetic_lut4(path, seed=9, centroid_layout=layout, **cfg)
    gpu = g.load_genomic_auto(path, device=0, max_ctx=128)
    assert gpu.info().megakernel == 0
    ref = O.OracleModel(path)
    gpu.set_k_wta_ratio(0.0)
    ref.set_k_wta_ratio(0.0)
    prompt = [int(t) for t in np.random.default_rng(4).integers(0, gpu.vocab_size, 12)]
    worst = 0.0
    for i, t in enumerate(prompt):
        worst = max(worst, _rel(gpu.forward(t, i == 0), lr := ref.forward(t, i == 0)))
    tok = int(np.argmax(lr))
    for _ in range(64):
        lg, lr = gpu.forward(tok), ref.forward(tok)
        worst = max(worst, _rel(lg, lr))
        assert int(np.argmax(lg)) == int(np.argmax(lr))
        tok = int(np.argmax(lr))
    assert worst <= REL_TOL, worst
    gpu.close()


def test_lut4_mixed_with_q4(g, O, tmp_path):
    """Only attn_output and ffn_down as tables, the rest Q4_0."""
    cfg = dict(g.configs.CONFIGS["small"])
    path = str(tmp_path / "mixed.flat")
    flat_numpy.write_synthetic_lut4(path, seed=3, lut_tensors=("attn_output", "ffn_down"), **cfg)
    gpu = g.load_genomic_auto(path, device=0, max_ctx=64)
    ref = O.OracleModel(path)
    gpu.set_k_wta_ratio(0.0)
    ref.set_k_wta_ratio(0.0)
    assert gpu.generate_native_py([5, 6, 7], 24, 0.0, 1.0, []) == ref.generate([5, 6, 7], 24, 0.0, 1.0, ())
    gpu.close()
