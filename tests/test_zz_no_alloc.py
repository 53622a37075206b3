"""gaje_cuda_attention_decode_static: the decode attention entry point that
allocates nothing (its scratch is a static device buffer), called through the
C ABI and compared with gaje_cuda_attention_decode on the same inputs.

Collected last (file name) so that it also runs after every other test has
used the library in this process; it passes alone in a fresh process too.
"""
import ctypes as C

import numpy as np
import pytest

GAJE_ERR_UNSUPPORTED = 5


def _lib(g):
    return g.lib()


def test_oversized_geometry_is_rejected(g):
    """256 + n_head*64*(head_dim+2)*4 bytes must fit the 1 MiB buffer: 64 heads
    of 256 dims need 4.3 MB.  The check precedes any CUDA call (no GPU needed)."""
    lib = _lib(g)
    dummy = C.c_void_p(16)
    st = lib.gaje_cuda_attention_decode_static(dummy, dummy, dummy, 10, 16, 64, 8, 256, dummy, None)
    assert st == GAJE_ERR_UNSUPPORTED
    msg = lib.gaje_cuda_last_error().decode()
    assert "1048576" in msg and "bytes of scratch" in msg


@pytest.mark.gpu
@pytest.mark.parametrize("ctx,nh,nkv,hd", [(1025, 14, 2, 64), (300, 12, 2, 128), (17, 9, 3, 64)])
def test_static_scratch_matches_workspace_entry_point(g, ctx, nh, nkv, hd):
    import torch

    lib = _lib(g)
    rng = np.random.default_rng(ctx + nh)
    stride = 1100
    q = torch.from_numpy(rng.standard_normal(nh * hd).astype(np.float32)).cuda()
    K = torch.from_numpy((rng.standard_normal((nkv, stride, hd)) * 0.5).astype(np.float32)).cuda()
    V = torch.from_numpy(rng.standard_normal((nkv, stride, hd)).astype(np.float32)).cuda()
    ref = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    args = (C.c_void_p(q.data_ptr()), C.c_void_p(K.data_ptr()), C.c_void_p(V.data_ptr()), ctx, stride, nh, nkv, hd)
    assert lib.gaje_cuda_attention_decode(*args, C.c_void_p(ref.data_ptr()), None) == 0
    torch.cuda.synchronize()
    outs = []
    for _ in range(2):  # two calls in a row: the counters come back to zero
        out = torch.full((nh * hd,), float("nan"), dtype=torch.float32, device="cuda")
        st = lib.gaje_cuda_attention_decode_static(*args, C.c_void_p(out.data_ptr()), None)
        assert st == 0, lib.gaje_cuda_last_error()
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    r = ref.cpu().numpy()
    for o in outs:
        np.testing.assert_allclose(o, r, rtol=1e-4, atol=2e-5)
