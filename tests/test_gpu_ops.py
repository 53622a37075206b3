"""Op-level parity on the GPU, through the C ABI, against the CPU oracle.

Tolerances: dequantised weights bit-exact; dot products within 1e-5 of the
row's magnitude sum (sum|w*x|), the bound the FP32 accumulation order allows
(the oracle uses the AVX2 8-lane order, the kernels a tree); K-WTA masks and
argmax indices exact.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SWEEP = [(896, 896), (4864, 896), (896, 4864), (8960, 1536), (1536, 8960)]


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _q4(O, N, K, seed, std=0.02):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N, K)) * std).astype(np.float32)
    return W, O.quantize_q4_0(W)


@pytest.mark.parametrize("N,K", SWEEP + [(2, 32), (7, 64)])
def test_dequant_bit_exact(g, O, N, K):
    _, blocks = _q4(O, N, K, N + K)
    m = g.Q4Matrix(blocks, N, K)
    out = torch.empty(N * K, dtype=torch.float32, device="cuda")
    m.dequant(out.data_ptr())
    torch.cuda.synchronize()
    ref = O.q4_0_dequant(blocks, fused=True)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_edge_blocks_bit_exact(g, O):
    from test_format import _edge_blocks

    w = _edge_blocks()
    blocks = O.quantize_q4_0(w)
    n = w.size // 32
    m = g.Q4Matrix(blocks, n, 32)
    out = torch.empty(w.size, dtype=torch.float32, device="cuda")
    m.dequant(out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), O.q4_0_dequant(blocks, True).view(np.uint32))


def _check_rows(got, ref, W_abs_x, rel=1e-5):
    tol = rel * W_abs_x + 1e-6
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} rows off, worst {np.max(np.abs(got - ref) - tol)}"


@pytest.mark.parametrize("N,K", SWEEP)
@pytest.mark.parametrize("M", [1, 3, 8, 15, 16, 17, 64, 100, 130])
def test_q4_gemv_matches_oracle(g, O, N, K, M):
    """M < 16: CUDA-core kernels (f32 products).  M >= 16: the tcgen05
    kernel, whose bf16 hi/lo splits of w and x carry each product to within
    3 * 2^-18 (< 1.2e-5) of its f32 value, hence the 2e-5 bound there."""
    W, blocks = _q4(O, N, K, 7 * N + K)
    rng = np.random.default_rng(M)
    X = rng.standard_normal((M, K)).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    m = g.Q4Matrix(blocks, N, K, bias=bias)
    x, y = _dev(X), torch.empty((M, N), dtype=torch.float32, device="cuda")
    m.gemv(x.data_ptr(), y.data_ptr(), M)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    deq = np.abs(O.q4_0_dequant(blocks, True).reshape(N, K))
    for i in range(M):
        ref = O.q4_0_gemv(blocks, X[i], N, K, bias=bias)
        _check_rows(got[i], ref, deq @ np.abs(X[i]), 2e-5 if M >= 16 else 1e-5)


def test_q4_gemv_reference_linear_kat(g, O):
    """src/nn/linear/tests.rs:8-100 on the device: rows i*0.1 / -i*0.1, x = 1."""
    row0 = np.arange(32, dtype=np.float32) * np.float32(0.1)
    blocks = np.concatenate([O.quantize_q4_0(row0), O.quantize_q4_0(-row0)])
    m = g.Q4Matrix(blocks, 2, 32)
    x = _dev(np.ones(32, np.float32))
    y = torch.empty(2, dtype=torch.float32, device="cuda")
    m.gemv(x.data_ptr(), y.data_ptr(), 1)
    torch.cuda.synchronize()
    for r in range(2):
        expected = float(np.sum(O.q4_0_dequant(blocks[r * 20:(r + 1) * 20], fused=False)))
        assert abs(float(y[r]) - expected) < 1e-4


def test_q4_gemv_flush_small_sums(g, O):
    """|sum| < 1e-6 -> 0 (genomic.rs:331-335), then +bias."""
    K = 64
    W = np.zeros((4, K), np.float32)
    W[1, :] = 1e-3
    blocks = O.quantize_q4_0(W)
    x = np.zeros(K, np.float32)
    x[0] = 5e-4  # row 1 dot = 5e-7 -> flushed
    bias = np.array([0.25, 0.5, 0.0, -1.0], np.float32)
    m = g.Q4Matrix(blocks, 4, K, bias=bias)
    xd, y = _dev(x), torch.empty(4, dtype=torch.float32, device="cuda")
    m.gemv(xd.data_ptr(), y.data_ptr(), 1)
    torch.cuda.synchronize()
    ref = O.q4_0_gemv(blocks, x, 4, K, bias=bias)
    assert np.array_equal(y.cpu().numpy(), ref)
    assert float(y[1]) == 0.5


@pytest.mark.parametrize("N,K", [(49152, 576), (151936, 896), (1000, 1536), (3, 8)])
def test_f32_gemv_argmax(g, O, N, K):
    rng = np.random.default_rng(N)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    Wd, xd = _dev(W), _dev(x)
    logits = torch.empty(N, dtype=torch.float32, device="cuda")
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    g.f32_gemv_argmax(Wd.data_ptr(), xd.data_ptr(), N, K, logits.data_ptr(), am.data_ptr())
    torch.cuda.synchronize()
    ref = O.f32_gemv(W, x)
    _check_rows(logits.cpu().numpy(), ref, np.abs(W) @ np.abs(x))
    assert int(am[0]) == int(np.argmax(logits.cpu().numpy()))


def test_argmax_first_index_on_ties_and_nan(g):
    """Strict `>` against -inf (llm/forward.rs:262-271): ties -> lowest index,
    NaN never wins, -0.0 == +0.0, all -inf -> 0."""
    K = 4
    cases = [
        ([1.0, 3.0, 3.0, 2.0], 1),
        ([float("nan"), 1.0, 1.0, float("nan")], 1),
        ([-0.0, 0.0, -1.0, -0.0], 0),
        ([float("-inf"), float("-inf"), float("nan"), float("-inf")], 0),
    ]
    for vals, want in cases:
        N = len(vals)
        W = np.zeros((N, K), np.float32)
        W[:, 0] = vals
        x = np.array([1.0, 0, 0, 0], np.float32)
        am = torch.zeros(1, dtype=torch.int32, device="cuda")
        Wd, xd = _dev(W), _dev(x)
        g.f32_gemv_argmax(Wd.data_ptr(), xd.data_ptr(), N, K, None, am.data_ptr())
        torch.cuda.synchronize()
        assert int(am[0]) == want, vals


@pytest.mark.parametrize("n,eps", [(576, 1e-5), (896, 1e-6), (1536, 1e-6), (7, 1e-6)])
def test_rms_norm(g, O, n, eps):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    xd, wd = _dev(x), _dev(w)
    g.rms_norm(xd.data_ptr(), wd.data_ptr(), eps, n, out.data_ptr())
    torch.cuda.synchronize()
    ref = O.rms_norm(x, w, eps)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-6, atol=1e-7)


def _attn_ref(O, q, K, V, ctx, nh, nkv, hd):
    """attention.rs:88-127 with the oracle's AVX2 dot; softmax in the same order."""
    G = nh // nkv
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    out = np.zeros(nh * hd, np.float32)
    for h in range(nh):
        g_ = h // G
        s = np.array([O.dot_f32(q[h * hd:(h + 1) * hd], K[g_, t]) * scale for t in range(ctx)], np.float32)
        e = np.exp(s - s.max()).astype(np.float32)
        inv = np.float32(1.0) / (np.float32(e.astype(np.float64).sum()) + np.float32(1e-12))
        out[h * hd:(h + 1) * hd] = ((e * inv)[:, None] * V[g_, :ctx]).astype(np.float64).sum(0)
    return out


@pytest.mark.parametrize("ctx", [1, 15, 16, 17, 100, 1024, 1025, 2304])
@pytest.mark.parametrize("nh,nkv,hd", [(14, 2, 64), (9, 3, 64), (12, 2, 128)])
def test_attention_decode(g, O, ctx, nh, nkv, hd):
    rng = np.random.default_rng(ctx * 131 + nh)
    stride = 2400
    q = rng.standard_normal(nh * hd).astype(np.float32)
    K = (rng.standard_normal((nkv, stride, hd)) * 0.5).astype(np.float32)
    V = rng.standard_normal((nkv, stride, hd)).astype(np.float32)
    qd, Kd, Vd = _dev(q), _dev(K), _dev(V)
    out = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    g.attention_decode(qd.data_ptr(), Kd.data_ptr(), Vd.data_ptr(), ctx, stride, nh, nkv, hd, out.data_ptr())
    torch.cuda.synchronize()
    ref = _attn_ref(O, q, K, V, ctx, nh, nkv, hd)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("n,k", [(151936, 75968), (49152, 24576), (896, 448), (100, 1), (100, 99), (10, 10)])
def test_kwta_exact(g, O, n, k):
    rng = np.random.default_rng(n + k)
    s = rng.standard_normal(n).astype(np.float32)
    s[::7] = s[3]  # ties at and around the threshold
    d = _dev(s)
    g.kwta(d.data_ptr(), n, k)
    torch.cuda.synchronize()
    assert np.array_equal(d.cpu().numpy(), O.kwta(s, k))
