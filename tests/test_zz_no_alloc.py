"""ck_matvec_noalloc: the matvec entry point for callers that cannot allocate
device memory themselves (their device memory belongs to another caching
allocator, or their serving loop cannot absorb the device synchronisation of
cudaMalloc/cudaFree).  The test owns every buffer -- torch allocates the
inputs and outputs, as such a caller's allocator would -- and checks, on two
calls in a row, that the entry point gives what the allocating ck_matvec
gives, within the matvec tolerance of the parity suite.  The file name sorts
last so a run that stops at the first failure has run everything else."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MATVEC_TOL = 1e-4   # relative, as tests/test_gpu_parity.py::test_matvec


def _case(t, k, n, seed):
    import torch
    from chonklm_b200.quant import quantize
    g = torch.Generator().manual_seed(seed)
    data = quantize(torch.randn(n, k, generator=g) * 0.02, t)
    x = np.random.default_rng(seed).standard_normal(k).astype(np.float32)
    return data, x


def test_noalloc_matvec_matches_allocating_entry_point():
    import torch
    from chonklm_b200 import _lib
    from chonklm_b200.gguf import GGML_TYPE
    cases = [(GGML_TYPE.Q4_K, 1024, 3072, 1), (GGML_TYPE.Q6_K, 3072, 1024, 2)]   # two calls in a row
    for t, k, n, seed in cases:
        data, x = _case(t, k, n, seed)
        w_dev = torch.from_numpy(np.frombuffer(data, dtype=np.uint8).copy()).cuda()
        x_dev = torch.from_numpy(x).cuda()
        y_dev = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        _lib.matvec_noalloc(t, w_dev.data_ptr(), len(data), k, n, x_dev.data_ptr(), y_dev.data_ptr(), 0)
        got = y_dev.cpu().numpy()
        want = _lib.matvec(t, data, k, n, x)
        err = float(np.abs(got - want).max() / np.abs(want).max())
        assert err < MATVEC_TOL, (t, err)


def test_noalloc_rejects_oversize_weights():
    import torch
    from chonklm_b200 import _lib
    from chonklm_b200.gguf import GGML_TYPE
    k, n = 1024, 40000          # 40000 x 576 B = 23 MB > the 16 MiB static scratch
    w_dev = torch.zeros(n * 576, dtype=torch.uint8, device="cuda")
    x_dev = torch.zeros(k, dtype=torch.float32, device="cuda")
    y_dev = torch.zeros(n, dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.CkError, match="static scratch"):
        _lib.matvec_noalloc(GGML_TYPE.Q4_K, w_dev.data_ptr(), n * 576, k, n, x_dev.data_ptr(), y_dev.data_ptr(), 0)
