"""The quantisers on the device (gaje_cuda_quantize_q4_0 / _q8_0) against the
host quantisers and the oracle's restatement of quantize_q4_0_native
(src/compute/quantize/python.rs:152-232): the bytes must be identical."""
import numpy as np
import pytest
import torch

from test_format import _edge_blocks

pytestmark = pytest.mark.gpu


def _special_blocks():
    """Blocks with infinities, NaN and the f16 limits around them."""
    b = []
    x = np.linspace(-1, 1, 32).astype(np.float32)
    y = x.copy()
    y[5] = np.nan
    b.append(y)
    y = x.copy()
    y[0] = np.inf
    b.append(y)
    y = x.copy()
    y[31] = -np.inf
    b.append(y)
    b.append(np.full(32, 65519.0, np.float32))
    b.append(np.full(32, 65520.0, np.float32))
    b.append(np.linspace(-6e-8, 6e-8, 32).astype(np.float32))
    b.append(np.zeros(32, np.float32))
    return np.concatenate(b)


def _run(g, w, q8):
    d = torch.from_numpy(w).cuda()
    out = torch.zeros(w.size // 32 * (34 if q8 else 20), dtype=torch.uint8, device="cuda")
    (g.quantize_q8_0_device if q8 else g.quantize_q4_0_device)(d.data_ptr(), w.size, out.data_ptr())
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("kind", ["random", "edges", "special", "large"])
@pytest.mark.parametrize("q8", [False, True], ids=["q4_0", "q8_0"])
def test_device_quantizer_bytes(g, O, kind, q8):
    if kind == "random":
        w = (np.random.default_rng(0).standard_normal(32 * 4097) * 0.02).astype(np.float32)
    elif kind == "edges":
        w = _edge_blocks()
    elif kind == "special":
        w = _special_blocks()
    else:  # a Qwen2-0.5B gate_up matrix: many tiles and a partial last tile
        w = (np.random.default_rng(1).standard_normal(9728 * 896 + 32 * 77) * 0.02).astype(np.float32)
    dev = _run(g, w, q8)
    host = np.frombuffer((g.quantize_q8_0_native if q8 else g.quantize_q4_0_native)(w.tobytes()), np.uint8)
    assert np.array_equal(dev, host)
    if kind != "special":  # the oracle restates the reference (finite inputs)
        assert np.array_equal(dev, (O.quantize_q8_0 if q8 else O.quantize_q4_0)(w))


def test_device_quantizer_argument_errors(g):
    w = torch.zeros(64, dtype=torch.float32, device="cuda")
    out = torch.zeros(64, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        g.quantize_q4_0_device(w.data_ptr(), 33, out.data_ptr())
    with pytest.raises(ValueError):
        g.quantize_q4_0_device(w.data_ptr() + 4, 32, out.data_ptr())
    with pytest.raises(ValueError):
        g.quantize_q8_0_device(w.data_ptr(), 32, out.data_ptr() + 1)
