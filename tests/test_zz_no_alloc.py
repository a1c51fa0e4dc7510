"""ms_q4_gemm_noalloc: the projection with its scratch in a fixed device array.

Some hosts cannot let a library call allocate device memory (a server that
reserved all of HBM for KV pages up front, or a latency-critical path where an
implicitly synchronising cudaMalloc is not allowed).  The entry point serves
them with a static array inside the library.  Called through the C-ABI and
compared with ms_q4_gemm on two calls in a row, within the Q4 GEMM tests'
own tolerance (relative RMSE 2e-5): rows above 8 run on the CUDA-core tiled
kernel there, on the tensor cores in ms_q4_gemm.  The file name puts it last
in collection; it also passes alone.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MS_ERR_CAPACITY = 4


def rel_rmse(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(((a - b) ** 2).mean()) / (np.sqrt((b ** 2).mean()) + 1e-12))


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


def noalloc(ctx, w, C, A, M, accumulate, stream):
    from mojostream_b200._lib import lib
    return lib().ms_q4_gemm_noalloc(ctx.h, w.h, ctypes.c_void_p(C.data_ptr()),
                                    ctypes.c_void_p(A.data_ptr()), M, accumulate, stream)


# (16, 2560, 2048) and (64, 2560, 2048): the context's k-split would overflow
# the static array; the call lowers it (10 -> 5 and 10 -> 2 k-segments)
@pytest.mark.parametrize("M,K,N", [(4, 2560, 2048), (8, 10240, 512), (1, 1024, 1024),
                                   (16, 1024, 1024), (16, 2560, 2048), (64, 2560, 2048)])
def test_noalloc_matches_q4_gemm_twice(ctx, torch_cuda, M, K, N):
    from mojostream_b200.runtime import Q4Weight, _stream
    torch = torch_cuda
    rng = np.random.default_rng(M * 131 + K + N)
    W = rng.integers(0, 256, size=(K, N // 2), dtype=np.uint8)
    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    w = Q4Weight(ctx, W, K, N, 0.0125)
    ref = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    w.gemm(A, ref)
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    for call in range(2):  # two calls in a row on the same static scratch
        C = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        ctx.check(noalloc(ctx, w, C, A, M, 0, _stream()))  # raises with the message
        torch.cuda.synchronize()
        got = C.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}"
        assert rel_rmse(got, ref) < 2e-5, f"call {call}"
    ctx.sync()  # no kernel timed out
    w.close()


def test_noalloc_accumulates(ctx, torch_cuda):
    from mojostream_b200.runtime import Q4Weight, _stream
    torch = torch_cuda
    rng = np.random.default_rng(5)
    M, K, N = 4, 2560, 1024
    W = rng.integers(0, 256, size=(K, N // 2), dtype=np.uint8)
    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    C0 = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).cuda()
    w = Q4Weight(ctx, W, K, N, 0.01)
    ref = C0.clone()
    w.gemm(A, ref, accumulate=True)
    C = C0.clone()
    ctx.check(noalloc(ctx, w, C, A, M, 1, _stream()))
    torch.cuda.synchronize()
    assert rel_rmse(C.cpu().numpy(), ref.cpu().numpy()) < 2e-5
    w.close()


def test_noalloc_rejects_plans_beyond_the_static_scratch(ctx, torch_cuda):
    # M 8, K 65536, N 2048: 52 k-segments x 128 tiles x 16 x 8 partial floats
    # (851968) exceed the 262144 of the static array
    from mojostream_b200.runtime import Q4Weight, _stream
    torch = torch_cuda
    K, N, M = 65536, 2048, 8
    W = np.full((K, N // 2), 0x88, dtype=np.uint8)
    w = Q4Weight(ctx, W, K, N, 0.01)
    A = torch.zeros((M, K), dtype=torch.float32, device="cuda")
    C = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    assert noalloc(ctx, w, C, A, M, 0, _stream()) == MS_ERR_CAPACITY
    w.close()
