"""qdec_matvec_noalloc: the matvec entry point for callers that cannot let the library allocate device memory
(an application whose GPU memory belongs to another allocator, or a decode loop that must not allocate while it
runs).  It must give exactly what qdec_matvec gives, call after call, from its fixed in-library scratch array.

This file is collected last on purpose (pytest orders files by name), so a run that stops at its first failure
has run every other test before this one."""
import numpy as np
import pytest

from helpers import random_blocks, to_dev


def test_oversize_request_is_rejected_before_any_device_work():
    import qdec

    cap = qdec.matvec_noalloc_max_bytes()
    cols = 17408
    n = cap // qdec.act_row_bytes(qdec.Q4_K, cols) + 1  # one column more than the scratch holds
    with pytest.raises(qdec.QdecError) as e:
        qdec.matvec_noalloc(qdec.Q4_K, 1, 16, cols, 1, n, 1)
    assert e.value.code == qdec.EINVAL and "scratch" in str(e.value)


@pytest.mark.gpu
@pytest.mark.parametrize("t", [12, 13, 14, 8, 2])
def test_noalloc_matches_matvec_on_two_calls(t):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qdec

    rows, cols = 300, 5120
    w = to_dev(random_blocks(t, rows, cols, seed=77 + t))
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # the scratch keeps the previous call's bytes: the second call must not see them
        x = to_dev(np.random.default_rng(call * 10 + t).standard_normal((4, cols)).astype(np.float32) * (1 + call))
        y_ref = torch.empty(4 * rows, dtype=torch.float32, device="cuda")
        y_new = torch.empty(4 * rows, dtype=torch.float32, device="cuda")
        qdec.matvec(t, w.data_ptr(), rows, cols, x.data_ptr(), 4, y_ref.data_ptr(), stream)
        qdec.matvec_noalloc(t, w.data_ptr(), rows, cols, x.data_ptr(), 4, y_new.data_ptr(), stream)
        torch.cuda.synchronize()
        a, b = y_ref.cpu().numpy(), y_new.cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"type {t}, call {call}"
