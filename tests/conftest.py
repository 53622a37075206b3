import importlib
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on the B200 box)")


@pytest.fixture(scope="session")
def g():
    """The product package (its Python face over libgaje_cuda.so)."""
    builder = importlib.import_module("gaje-semantic-compression_b200.build")
    builder.build()
    return importlib.import_module("gaje-semantic-compression_b200")


@pytest.fixture(scope="session")
def O():
    """The CPU oracle (the checker)."""
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


def _model(g, model_dir, name, seed, **over):
    cfg = dict(g.configs.CONFIGS[name])
    cfg.update(over)
    path = os.path.join(str(model_dir), f"{name}-{seed}-{abs(hash(tuple(sorted(over.items()))))}.flat")
    if not os.path.exists(path):
        g.write_synthetic(path, seed=seed, **cfg)
    return path


@pytest.fixture(scope="session")
def make_model(g, model_dir):
    def mk(name, seed=1, **over):
        return _model(g, model_dir, name, seed, **over)

    return mk
