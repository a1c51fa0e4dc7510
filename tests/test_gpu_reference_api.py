"""The reference-named adapter (mojostream_b200/reference_api.py) on the GPU:
matmul_q4_bpack_raw (src/linalg/kernels.mojo:201-267) in both of its forms
against the oracle.  The layer and sampling adapters are checked in
test_gpu_parity.py and test_gpu_sampler.py."""
import numpy as np
import pytest

from parity_util import rel_rmse, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def ctx(torch_cuda):
    from mojostream_b200.runtime import Context
    c = Context(0)
    yield c
    c.close()


def test_reference_named_q4_matmul_both_forms(ctx, torch_cuda, oracle_lib):
    """reference_api.matmul_q4_bpack_raw (kernels.mojo:201-267: C += A . W)
    given raw bytes (a one-off call: its own context, upload and repack) and
    given a Q4Weight made once (a host loop's form, called twice), both
    against the oracle; a scale other than the weight's is refused."""
    from mojostream_b200 import reference_api as ra
    from mojostream_b200.runtime import Q4Weight
    torch = torch_cuda
    rng = np.random.default_rng(3)
    K, N, M = 1024, 512, 4
    W = rng.integers(0, 256, size=(K, N // 2), dtype=np.uint8)
    A = rng.standard_normal((M, K)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    once = oracle_lib.q4_matmul(A, W, N, 0.01, C=C0)
    C = to_dev(torch, C0)
    ra.matmul_q4_bpack_raw(C, to_dev(torch, A), W, N // 2, 0.01)
    torch.cuda.synchronize()
    assert rel_rmse(C.cpu().numpy(), once) < 2e-5
    w = Q4Weight(ctx, W, K, N, 0.01)
    C = to_dev(torch, C0)
    for _ in range(2):
        ra.matmul_q4_bpack_raw(C, to_dev(torch, A), w, N // 2, 0.01)
    torch.cuda.synchronize()
    twice = oracle_lib.q4_matmul(A, W, N, 0.01, C=once)
    assert rel_rmse(C.cpu().numpy(), twice) < 2e-5
    with pytest.raises(ValueError, match="scale"):
        ra.matmul_q4_bpack_raw(C, to_dev(torch, A), w, N // 2, 0.02)
    w.close()
