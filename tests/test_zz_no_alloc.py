"""gaje_cuda_attention_decode_static: the decode attention entry point that
allocates nothing (its scratch is a static device buffer), called through the
C ABI and compared with gaje_cuda_attention_decode and with the oracle's
attention on the same inputs.

Some hosts cannot allocate device memory once they are serving: a caller that
budgets all of its device memory at start-up, or one that cannot afford the
device-wide synchronisation a cudaMalloc/cudaFree brings.  This entry point is
for them.

Collected last (file name) so that it also runs after every other test has
used the library in this process; it passes alone in a fresh process too.
"""
import ctypes as C

import numpy as np
import pytest

GAJE_ERR_INVALID = 1
GAJE_ERR_UNSUPPORTED = 5


def _lib(g):
    return g.lib()


def test_oversized_geometry_is_rejected(g):
    """512 + n_head*64*(head_dim+2)*4 bytes must fit the 1 MiB buffer: 64 heads
    of 256 dims need 4.3 MB.  The check precedes any CUDA call (no GPU needed)."""
    lib = _lib(g)
    dummy = C.c_void_p(16)
    st = lib.gaje_cuda_attention_decode_static(dummy, dummy, dummy, 10, 16, 64, 8, 256, dummy, None)
    assert st == GAJE_ERR_UNSUPPORTED
    msg = lib.gaje_cuda_last_error().decode()
    assert "1048576" in msg and "bytes of scratch" in msg


@pytest.mark.parametrize("entry", ["gaje_cuda_attention_decode", "gaje_cuda_attention_decode_static"])
@pytest.mark.parametrize("which", [0, 1, 2, 3])
def test_misaligned_pointers_are_rejected(g, entry, which):
    """The cache rows are bulk-copied (16-byte aligned sources only): a pointer
    off a 16-byte boundary is an argument error before any CUDA call."""
    lib = _lib(g)
    ptrs = [C.c_void_p(4096) for _ in range(4)]
    ptrs[which] = C.c_void_p(4096 + 4)
    q, k, v, out = ptrs
    st = getattr(lib, entry)(q, k, v, 10, 16, 14, 2, 64, out, None)
    assert st == GAJE_ERR_INVALID
    assert "16-byte aligned" in lib.gaje_cuda_last_error().decode()


def _oracle_attention(O, q, K, V, ctx, nh, nkv, hd):
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


@pytest.mark.gpu
@pytest.mark.parametrize("ctx,nh,nkv,hd", [(1025, 14, 2, 64), (300, 12, 2, 128), (17, 9, 3, 64), (5, 14, 2, 64)])
def test_static_scratch_matches_workspace_entry_point(g, O, ctx, nh, nkv, hd):
    """Two calls in a row (the counters come back to zero in between) equal the
    workspace entry point and the oracle.  ctx 5 runs a single split, which
    writes its output directly and never touches the counters."""
    import torch

    lib = _lib(g)
    rng = np.random.default_rng(ctx + nh)
    stride = 1100
    qh = rng.standard_normal(nh * hd).astype(np.float32)
    Kh = (rng.standard_normal((nkv, stride, hd)) * 0.5).astype(np.float32)
    Vh = rng.standard_normal((nkv, stride, hd)).astype(np.float32)
    q, K, V = (torch.from_numpy(a).cuda() for a in (qh, Kh, Vh))
    ref = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    args = (C.c_void_p(q.data_ptr()), C.c_void_p(K.data_ptr()), C.c_void_p(V.data_ptr()), ctx, stride, nh, nkv, hd)
    assert lib.gaje_cuda_attention_decode(*args, C.c_void_p(ref.data_ptr()), None) == 0
    torch.cuda.synchronize()
    outs = []
    for _ in range(2):
        out = torch.full((nh * hd,), float("nan"), dtype=torch.float32, device="cuda")
        st = lib.gaje_cuda_attention_decode_static(*args, C.c_void_p(out.data_ptr()), None)
        assert st == 0, lib.gaje_cuda_last_error()
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    r = ref.cpu().numpy()
    oracle = _oracle_attention(O, qh, Kh, Vh, ctx, nh, nkv, hd)
    for o in outs:
        np.testing.assert_allclose(o, r, rtol=1e-4, atol=2e-5)
        np.testing.assert_allclose(o, oracle, rtol=1e-4, atol=2e-5)


@pytest.mark.gpu
def test_static_entry_point_allocates_no_device_memory(g):
    """After the first call on the device (which looks the buffer up and may
    load the module), further calls leave the device's free memory unchanged."""
    import torch

    lib = _lib(g)
    nh, nkv, hd, ctx, stride = 14, 2, 64, 700, 800
    rng = np.random.default_rng(3)
    q = torch.from_numpy(rng.standard_normal(nh * hd).astype(np.float32)).cuda()
    K = torch.from_numpy(rng.standard_normal((nkv, stride, hd)).astype(np.float32)).cuda()
    V = torch.from_numpy(rng.standard_normal((nkv, stride, hd)).astype(np.float32)).cuda()
    outs = [torch.empty(nh * hd, dtype=torch.float32, device="cuda") for _ in range(3)]
    args = (C.c_void_p(q.data_ptr()), C.c_void_p(K.data_ptr()), C.c_void_p(V.data_ptr()), ctx, stride, nh, nkv, hd)
    assert lib.gaje_cuda_attention_decode_static(*args, C.c_void_p(outs[0].data_ptr()), None) == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for o in outs[1:]:
        assert lib.gaje_cuda_attention_decode_static(*args, C.c_void_p(o.data_ptr()), None) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.equal(outs[1], outs[0]) and torch.equal(outs[2], outs[0])
