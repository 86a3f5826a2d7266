"""The allocation-free C entry point (``br_muon_normalize_noalloc``) against the library's list-based
Muon momentum + normalisation entry point.

The entry point is for callers that cannot allocate device memory (memory-planned runtimes, host code
that must not call cudaMalloc); it keeps its scratch in a fixed array inside the library. This test
calls it through its exported C symbol, twice in a row with different inputs (the second call must not
see the first call's scratch), and checks both the normalised update and the in-place momentum
against ``muon_prepare``. It lives in its own file, collected after every other test, and passes both
alone in a fresh process and after the rest of the suite.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

CUDA_ERROR_INVALID_VALUE = 1


def _entry():
    from bitresearch_b200 import _C  # loads the library; ctypes then resolves the C symbol in it
    lib = ctypes.CDLL(_C.__file__)
    f = lib.br_muon_normalize_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                  ctypes.c_void_p]
    return f


def test_noalloc_entry_matches_list_entry(cuda):
    from bitresearch_b200.ops._ext import ext
    f = _entry()
    torch.manual_seed(0)
    S, r, c = 6, 512, 256
    n = r * c
    mu = 0.9
    mom_a = torch.randn(S, r, c, device=cuda) * 0.01  # state advanced by the C entry point
    mom_b = mom_a.clone()                             # state advanced by the list entry point
    xa = torch.empty(S, r, c, dtype=torch.bfloat16, device=cuda)
    xb = torch.empty_like(xa)
    ss = torch.empty(ext().muon_prepare_scratch(S, n), device=cuda)  # the list entry point's scratch
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for call in range(2):
        g = torch.randn(S, r, c, device=cuda) * (0.01 * (call + 1))
        rc = f(g.data_ptr(), mom_a.data_ptr(), xa.data_ptr(), S, n, mu, stream)
        assert rc == 0
        ext().muon_prepare([g[i] for i in range(S)], [mom_b[i] for i in range(S)], mu, xb, ss)
        torch.cuda.synchronize()
        torch.testing.assert_close(mom_a, mom_b, rtol=1e-6, atol=1e-7)
        err = (xa.float() - xb.float()).abs().max().item()
        assert err <= 1e-2 * xb.float().abs().max().item(), (call, err)
        # each matrix is normalised to Frobenius norm 1/1.02
        norms = xa.float().flatten(1).norm(dim=1)
        assert torch.allclose(norms, torch.full_like(norms, 1 / 1.02), rtol=1e-2)


def test_noalloc_entry_rejects_sizes_beyond_its_scratch(cuda):
    f = _entry()
    x = torch.empty(8, device=cuda)
    xb = torch.empty(8, dtype=torch.bfloat16, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    assert f(x.data_ptr(), x.data_ptr(), xb.data_ptr(), 4097, 1, 0.9, stream) == CUDA_ERROR_INVALID_VALUE
    assert f(x.data_ptr(), x.data_ptr(), xb.data_ptr(), 0, 1, 0.9, stream) == CUDA_ERROR_INVALID_VALUE
    assert f(None, x.data_ptr(), xb.data_ptr(), 1, 8, 0.9, stream) == CUDA_ERROR_INVALID_VALUE
