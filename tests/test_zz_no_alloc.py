"""hg_op_q8_matvec_noalloc, the Q8 matvec for callers that cannot allocate device memory (for
example a host framework whose pool already holds all free device memory, or a serving thread
that must not block on driver allocation calls). It uses a fixed scratch array compiled into the
library instead of allocating, so its results must equal hg_op_q8_matvec's bit for bit. This file
is collected last so a failure here comes after every other test has run."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _pack(native, w):
    rows, cols = w.shape
    ss = native.lib().hg_q8_scale_stride(cols)
    qs = np.empty((rows, cols), np.int8)
    sc = np.empty((rows, ss), np.float32)
    native.check(native.lib().hg_q8_pack(w.ctypes.data, rows, cols, qs.ctypes.data, sc.ctypes.data))
    return qs, sc


def _run(native, fn, rows, cols, ntok, seed):
    import torch

    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    qs, sc = _pack(native, w)
    dq, ds, dx = _dev(qs), _dev(sc), _dev(x)
    dy = torch.full((ntok, rows), float("nan"), dtype=torch.float32, device="cuda")
    native.check(fn(dq.data_ptr(), ds.data_ptr(), rows, cols, dx.data_ptr(), dy.data_ptr(), ntok, None))
    torch.cuda.synchronize()
    return dy.cpu().numpy()


@pytest.mark.parametrize("calls", [
    ((2304, 768, 3, 11), (768, 1536, 17, 12)),   # small, then large
    ((768, 1536, 17, 13), (2304, 768, 1, 14)),   # large, then small: stale bytes from the first
                                                 # call lie where the second reads its scales
    ((320, 768, 1, 15), (768, 320, 1, 16)),      # one token per call (the single-token kernel)
])
def test_noalloc_matches_allocating_matvec_on_two_calls(native, calls):
    lib = native.lib()
    # two calls in a row share the scratch array; the second must not see the first's contents
    for rows, cols, ntok, seed in calls:
        got = _run(native, lib.hg_op_q8_matvec_noalloc, rows, cols, ntok, seed)
        ref = _run(native, lib.hg_op_q8_matvec, rows, cols, ntok, seed)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (rows, cols, ntok)


def test_noalloc_rejects_sizes_beyond_its_scratch(native):
    lib = native.lib()
    cols, ntok = 8192, 1024  # 8 MiB of int8 activations > the 4 MiB array
    assert ntok * cols > native.NOALLOC_SCRATCH_BYTES
    rc = lib.hg_op_q8_matvec_noalloc(C.c_void_p(16), C.c_void_p(16), 64, cols, C.c_void_p(16), C.c_void_p(16),
                                     ntok, None)
    assert rc == -1
    assert b"scratch" in lib.hg_last_error()
