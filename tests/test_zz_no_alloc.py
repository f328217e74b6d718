"""The allocation-free argmax entry point, called through the C ABI.

It serves hosts that own all device memory themselves and cannot let the library
allocate during the token loop.  The test hands it device buffers (allocated here
by the test, as such a host would from its own pool) and checks its indices
against the allocating entry point llmdot_cuda_argmax and against the CPU oracle's
restatement of the reference's ArgMax on two calls in a row: the second call uses
smaller logits and more rows, so keys left over from the first call would win if
the entry point did not clear them.  Rows with NaN, signed zeros and infinities
check that it returns what the reference's strict-`>` scan returns.  Index results
are compared exactly (the tolerance used for argmax everywhere in these tests).

The file is named so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call(lib, x_dev, n, rows, ld, idx_dev):
    return lib.llmdot_cuda_argmax_noalloc(C.c_void_p(x_dev), n, rows, ld, C.c_void_p(idx_dev), None)


def test_argmax_noalloc_matches_allocating_entry_point(backend, oracle):
    import torch
    from dotllm_b200 import native

    lib = native.lib()
    rng = np.random.default_rng(1234)
    for call, (rows, n, scale) in enumerate([(3, 128256, 10.0), (8, 32000, 1.0)]):
        x = (rng.standard_normal((rows, n)) * scale).astype(np.float32)
        x[1, 7] = x[1, n - 9] = x[1].max() + 1.0  # tie: the lowest index wins
        x[2, 0] = np.float32("nan")  # a NaN at element 0 is never replaced
        if rows > 3:
            x[3, 11] = np.float32("nan")  # a NaN elsewhere never wins
            x[4, :] = -1.0
            x[4, 5], x[4, 9] = -0.0, 0.0  # -0 and +0 are equal: the first stays
            x[5, n - 2] = np.float32("inf")
        dx = torch.from_numpy(x).to("cuda:0")
        di = torch.full((rows,), -1, dtype=torch.int32, device="cuda:0")
        torch.cuda.synchronize()
        rc = _call(lib, dx.data_ptr(), n, rows, n, di.data_ptr())
        assert rc == 0, lib.llmdot_cuda_last_error().decode()
        torch.cuda.synchronize()
        got = di.cpu().numpy().tolist()
        want = [backend.arg_max(x[r]) for r in range(rows)]
        assert got == want, f"call {call + 1}: {got} != {want}"
        assert got == [oracle.argmax(x[r]) for r in range(rows)], f"call {call + 1}: differs from the oracle"
        assert got[1] == 7 and got[2] == 0


def test_argmax_noalloc_rejects_rows_beyond_its_scratch(gpu):
    import torch
    from dotllm_b200 import native

    lib = native.lib()
    limit = 4096  # LLMDOT_ARGMAX_NOALLOC_MAX_ROWS
    dx = torch.zeros((limit + 1) * 8, dtype=torch.float32, device="cuda:0")
    di = torch.zeros(limit + 1, dtype=torch.int32, device="cuda:0")
    rc = _call(lib, dx.data_ptr(), 8, limit + 1, 8, di.data_ptr())
    assert rc == -1
    assert "exceeds the fixed scratch" in lib.llmdot_cuda_last_error().decode()
    assert _call(lib, 0, 8, 1, 8, di.data_ptr()) == -1
