"""Failure handling of the bounded device waits, on one GPU, without a peer and without a fault: each wait is
made to run into its limit by data that never arrives (a flag nothing sets), must give up with its error word,
and must leave the context usable -- the same work run normally afterwards gives the right result.

  - the tensor-parallel exchange poll: the peer's lines carry the previous step's tag, so the step's tag never
    shows; the slot's error word 0x10000 | slot is recorded;
  - the decode GEMV's stage wait: the first window's barrier expects 16 bytes more than its copies bring.

The waits the engine runs report the same words through qdec_state_sync as QDEC_ETIMEOUT."""
import time

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def q():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qdec

    return qdec


@pytest.mark.parametrize("which", [0, 1], ids=["exchange_poll", "gemv_stage_wait"])
def test_bounded_wait_gives_up_and_context_stays_usable(q, which):
    t0 = time.time()
    q.selftest_wait(which, 200)
    dt = time.time() - t0
    assert dt >= 0.2, f"the wait returned after {dt:.3f} s, before its 0.2 s limit"
    assert dt < 30, dt
    # the context is still usable: an ordinary library call afterwards
    x = torch.randn(256, device="cuda")
    out = torch.empty(320, dtype=torch.uint8, device="cuda")
    q.quantize_image(12, x.data_ptr(), 256, 1, out.data_ptr(), 0)
    torch.cuda.synchronize()


def test_selftest_rejects_bad_arguments(q):
    with pytest.raises(q.QdecError) as e:
        q.selftest_wait(2, 100)
    assert e.value.code == q.EINVAL
    with pytest.raises(q.QdecError):
        q.selftest_wait(0, 0)
