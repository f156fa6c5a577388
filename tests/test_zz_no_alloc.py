"""The allocation-free entry point, pfng_b200_compute_q4_0_noalloc (GPU).

Some callers cannot allocate device memory where they call the matmul (a
server whose pool owns the whole GPU, a loop that cannot take cudaMalloc's
synchronisation).  This entry point keeps its scratch in a fixed 16 MiB array
inside the library instead of a caller workspace.  On two calls in a row of
different shapes sharing that scratch -- one large enough for a single pass
over k, one small-m shape whose k is split across CTAs -- its C must be
bit-identical to pfng_b200_compute_q4_0 on the tensor-core path and within
the reference's tolerance of the oracle; a problem whose scratch would not
fit must be refused before anything is launched.

The file is named to be collected last, and its first call also performs the
per-device set-up, so it passes both alone and after the other tests.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import pfng_b200 as pb  # noqa: E402

TOL = 1e-5


def _noalloc():
    f = pb.lib().pfng_b200_compute_q4_0_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    return f


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    yield


def _case(oracle, m, n, k, seed):
    rng = np.random.default_rng(seed)
    w = oracle.quantize("q4_0", rng.standard_normal((n, k)).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = oracle.quantize("q8_0", x)
    wd = torch.from_numpy(w.view(np.uint8).reshape(-1).copy()).cuda()
    xd = torch.from_numpy(x).cuda()
    return w, a, wd, xd, oracle.bound("q4_0", w, a, m, n, k)


def test_noalloc_matches_compute_on_two_calls(oracle):
    f = _noalloc()
    stream = torch.cuda.current_stream().cuda_stream
    for m, n, k, seed in ((130, 300, 1536, 1), (32, 4096, 4096, 2)):
        w, a, wd, xd, bound = _case(oracle, m, n, k, seed)
        c = torch.full((m, n), float("nan"), device="cuda")
        st = f(wd.data_ptr(), xd.data_ptr(), xd.stride(0), c.data_ptr(), m, n, k, c.stride(0), stream)
        assert st == 0, pb.status_string(st)
        same = pb.compute("q4_0", wd, xd, n, path="mma")
        torch.cuda.synchronize()
        got = c.cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), same.cpu().numpy().view(np.uint32))
        ref = oracle.mm("q4_0", w, a, m, n, k)
        err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        assert np.all(err <= TOL * bound + 1e-30), f"max error {err.max()} at m={m} n={n} k={k}"
    pb.check_kernel_error()


def test_noalloc_rejects_problems_beyond_its_scratch():
    f = _noalloc()
    # 4096 rows of k = 11008 need ~56 MiB of scratch: refused on the host
    st = f(0x10000, 0x10000, 11008, 0x10000, 4096, 64, 11008, 64, None)
    assert st == -4
