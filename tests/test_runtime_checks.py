"""The Python wrappers hand tensors to the C-ABI as bare pointers, so they
check what the library cannot see (device, dtype, layout, size) before the
call; checked here without a GPU through a stand-in tensor."""
import pytest
import torch

from mojostream_b200.runtime import _check_f32


class FakeCuda:
    """What _check_f32 reads of a CUDA tensor."""

    def __init__(self, n, dtype=torch.float32, contiguous=True):
        self.is_cuda, self.dtype, self._c, self._n = True, dtype, contiguous, n

    def is_contiguous(self):
        return self._c

    def numel(self):
        return self._n


def test_accepts_a_dense_f32_cuda_tensor_of_enough_values():
    _check_f32(FakeCuda(12), "x", 12)
    _check_f32(FakeCuda(13), "x", 12)


@pytest.mark.parametrize("t,needle", [
    (torch.zeros(12), "CUDA tensor"),
    (FakeCuda(12, dtype=torch.bfloat16), "float32 needed"),
    (FakeCuda(12, contiguous=False), "contiguous"),
    (FakeCuda(11), "11 values, the call uses 12"),
])
def test_rejects_what_the_library_would_misread(t, needle):
    with pytest.raises(ValueError, match=needle):
        _check_f32(t, "x", 12)


def test_reference_matmul_refuses_a_mismatched_prebuilt_weight():
    """reference_api.matmul_q4_bpack_raw with a Q4Weight made once: a weight
    of another shape or scale is refused before any launch."""
    from mojostream_b200 import reference_api as ra
    from mojostream_b200.runtime import Q4Weight
    w = object.__new__(Q4Weight)  # the fields the call checks; no device weight
    w.K, w.N, w.scale, w.h = 64, 32, 0.01, None
    A, C = torch.zeros((2, 64)), torch.zeros((2, 32))
    with pytest.raises(ValueError, match="scale"):
        ra.matmul_q4_bpack_raw(C, A, w, 16, 0.02)
    with pytest.raises(ValueError, match="weight is 64 x 32"):
        ra.matmul_q4_bpack_raw(torch.zeros((2, 64)), A, w, 32, 0.01)
    with pytest.raises(ValueError, match="C is"):
        ra.matmul_q4_bpack_raw(torch.zeros((3, 32)), A, w, 16, 0.01)


def test_row_lists_must_match_the_row_count():
    from mojostream_b200.runtime import _check_rows
    _check_rows(3, seq=[0, 0, 1], pos=[4, 5, 0])
    with pytest.raises(ValueError, match="pos: 2 entries for 3 rows"):
        _check_rows(3, seq=[0, 0, 1], pos=[4, 5])


def test_reference_matmul_raw_form_call_sequence(monkeypatch):
    """matmul_q4_bpack_raw given raw bytes: it makes its own context, uploads
    the weight, launches with accumulation, waits on the launching stream and
    closes both, in that order (stand-ins for the library objects)."""
    import numpy as np

    from mojostream_b200 import reference_api as ra
    calls = []

    class Ctx:
        def __init__(self, device=0):
            calls.append(("ctx", device))

        def sync(self, current=False):
            calls.append(("sync", current))

        def close(self):
            calls.append(("ctx.close",))

    class W:
        def __init__(self, ctx, w, K, N, scale):
            calls.append(("weight", w.shape, K, N, scale))

        def gemm(self, A, C, accumulate=False):
            calls.append(("gemm", tuple(A.shape), tuple(C.shape), accumulate))

        def close(self):
            calls.append(("weight.close",))

    monkeypatch.setattr(ra.runtime, "Context", Ctx)
    monkeypatch.setattr(ra.runtime, "Q4Weight", W)
    A, C = torch.zeros((4, 64)), torch.zeros((4, 32))
    bq = np.zeros((64, 16), np.uint8)
    assert ra.matmul_q4_bpack_raw(C, A, bq, 16, 0.01) is C
    assert calls == [("ctx", 0), ("weight", (64, 16), 64, 32, 0.01),
                     ("gemm", (4, 64), (4, 32), True), ("sync", True), ("weight.close",),
                     ("ctx.close",)]
