import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def tiny_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("tiny_models"))


_cache = {}


def tiny_model(tiny_dir: str, arch: str, quant: str = "q4_k_m", **kw) -> str:
    """Seeded tiny GGUF (generated once per session, on the CPU so the bytes
    are the same on every machine)."""
    from chonklm_b200.synth import tiny_spec, write_synthetic_gguf
    key = (arch, quant, tuple(sorted(kw.items())))
    if key not in _cache:
        name = f"tiny_{arch}_{quant}" + "".join(f"_{k}{v}" for k, v in sorted(kw.items())) + ".gguf"
        path = os.path.join(tiny_dir, name)
        write_synthetic_gguf(tiny_spec(arch, quant, **kw), path, seed=0, device="cpu")
        _cache[key] = path
    return _cache[key]
