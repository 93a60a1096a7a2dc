"""ck_matvec_noalloc: the matvec entry point for callers that cannot allocate
device memory themselves -- their device memory belongs to another caching
allocator (a framework pool that already holds the GPU's memory), or their
serving loop cannot absorb the device synchronisation of cudaMalloc/cudaFree.

The test owns every buffer (torch allocates the inputs and outputs, as such a
caller's allocator would) and checks, on two calls in a row, that the entry
point gives what the fp64 oracle and the allocating ck_matvec give, within
the matvec tolerance of the parity suite; that it runs on a caller's own
stream; and that once a device is set up, a call leaves the device's free
memory unchanged.  The file name sorts last so a run that stops at the first
failure has run everything else."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MATVEC_TOL = 1e-4   # relative (max |d| / max |want|), as tests/test_gpu_parity.py::test_matvec


def _case(t, k, n, seed):
    import torch
    from chonklm_b200.quant import quantize
    g = torch.Generator().manual_seed(seed)
    data = quantize(torch.randn(n, k, generator=g) * 0.02, t)
    x = np.random.default_rng(seed).standard_normal(k).astype(np.float32)
    return data, x


def _rel(got, want):
    return float(np.abs(got - want).max() / np.abs(want).max())


def test_noalloc_matvec_matches_oracle_and_allocating_entry_point():
    import torch
    from chonklm_b200 import _lib
    from chonklm_b200.gguf import GGML_TYPE
    from oracle import oracle
    cases = [(GGML_TYPE.Q4_K, 1024, 3072, 1), (GGML_TYPE.Q6_K, 3072, 1024, 2)]   # two calls in a row
    for t, k, n, seed in cases:
        data, x = _case(t, k, n, seed)
        w_dev = torch.from_numpy(np.frombuffer(data, dtype=np.uint8).copy()).cuda()
        x_dev = torch.from_numpy(x).cuda()
        y_dev = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        _lib.matvec_noalloc(t, w_dev.data_ptr(), len(data), k, n, x_dev.data_ptr(), y_dev.data_ptr(), 0)
        got = y_dev.cpu().numpy()
        truth = oracle.matvec(t, np.frombuffer(data, np.uint8), k, n, x, oracle.MODE_F64)
        assert _rel(got, truth) < MATVEC_TOL, (t, "oracle", _rel(got, truth))
        want = _lib.matvec(t, data, k, n, x)
        assert _rel(got, want) < MATVEC_TOL, (t, "ck_matvec", _rel(got, want))


def test_noalloc_on_caller_stream_allocates_nothing():
    import torch
    from chonklm_b200 import _lib
    from chonklm_b200.gguf import GGML_TYPE
    from oracle import oracle
    t, k, n = GGML_TYPE.Q4_K, 2048, 1536
    data, x = _case(t, k, n, 3)
    w_dev = torch.from_numpy(np.frombuffer(data, dtype=np.uint8).copy()).cuda()
    x_dev = torch.from_numpy(x).cuda()
    y_dev = torch.zeros(n, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    # first call: the device's one-time set-up (and the kernels' first load)
    _lib.matvec_noalloc(t, w_dev.data_ptr(), len(data), k, n, x_dev.data_ptr(), y_dev.data_ptr(), s.cuda_stream)
    truth = oracle.matvec(t, np.frombuffer(data, np.uint8), k, n, x, oracle.MODE_F64)
    assert _rel(y_dev.cpu().numpy(), truth) < MATVEC_TOL
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    y_dev.fill_(float("nan"))
    torch.cuda.synchronize()
    _lib.matvec_noalloc(t, w_dev.data_ptr(), len(data), k, n, x_dev.data_ptr(), y_dev.data_ptr(), s.cuda_stream)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert _rel(y_dev.cpu().numpy(), truth) < MATVEC_TOL


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
