"""Failure detection on the GPU without a fault (GPU).

Every pipelined kernel of the library waits on mbarriers with a bounded
wait; a wait that runs out records an error in the library's device error
word and the kernel returns, so the context stays usable and the host learns
of it from pfng_b200_check_kernel_error (PFNG_B200_ERR_KERNEL_TIMEOUT, -6).
The reference has no device code; its failure convention is fail-closed
(bench/framework/kernel_registry.cpp:13-17: a bad registration aborts, a
failed prepare or export is a FAIL with a message).

Here the wait is made to run out on purpose: pfng_b200_selftest_wait runs a
producer warp that skips its arrive and a consumer that waits through the
same bounded-wait helper with a limit of a few thousand ~1 us tries.  The
test checks the reported status, that the error word is cleared by the read,
and that the next real matmul on the same context succeeds and is correct.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import pfng_b200 as pb  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    pb.check_kernel_error()  # start from a clear error word
    yield


def test_wait_that_completes_reports_nothing():
    done, status = pb.selftest_wait(4096, skip_arrive=False)
    assert done == 1 and status == pb.OK


def test_wait_that_runs_out_reports_timeout_and_context_survives(oracle):
    done, status = pb.selftest_wait(2000, skip_arrive=True)
    assert done == 0
    assert status == pb.ERR_KERNEL_TIMEOUT
    # the read cleared the word
    assert pb.lib().pfng_b200_check_kernel_error(None) == pb.OK
    # the context is still usable: a real matmul right after is correct
    rng = np.random.default_rng(9)
    m, n, k = 3, 256, 1024
    w = oracle.quantize("q4_0", rng.standard_normal((n, k)).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = oracle.quantize("q8_0", x)
    wd = torch.from_numpy(w.view(np.uint8).reshape(-1).copy()).cuda()
    c = pb.compute("q4_0", wd, torch.from_numpy(x).cuda(), n)
    torch.cuda.synchronize()
    err = np.abs(c.cpu().numpy().astype(np.float64) - oracle.mm("q4_0", w, a, m, n, k))
    assert np.all(err <= 1e-5 * oracle.bound("q4_0", w, a, m, n, k) + 1e-30)
    pb.check_kernel_error()
