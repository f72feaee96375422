"""CPU-side checks of the C ABI: the library loads without a GPU, exports every symbol include/qdec.h
declares, and rejects bad arguments (the reference's assert! conditions) before touching the device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "qdec.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qdec_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def q():
    import qdec

    return qdec


def test_library_exports_every_declared_symbol(q):
    L = q.lib()
    names = declared_symbols()
    assert len(names) >= 8
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/qdec.h but not exported"


def test_version(q):
    assert q.version().startswith("qdec ")


def test_bad_shapes_rejected_without_gpu(q):
    with pytest.raises(q.QdecError) as e:
        q.gemv(q.Q4_K, 1, 10, 300, 1, 1, 1)  # cols not a multiple of 256
    assert e.value.code == q.EINVAL and "multiple" in str(e.value)
    with pytest.raises(q.QdecError):
        q.gemv(99, 1, 10, 256, 1, 1, 1)  # unsupported type
    with pytest.raises(q.QdecError):
        q.quantize_q8k(1, 100, 1, 1)
    with pytest.raises(q.QdecError):
        q.gemv(q.Q8_0, 1, 10, 32, 1, 1, 1)  # odd number of 32-blocks
    with pytest.raises(q.QdecError):
        q.gemv(q.Q4_K, 0, 10, 256, 1, 1, 1)  # null weights


def test_act_row_bytes(q):
    assert q.act_row_bytes(q.Q4_K, 5120) == 20 * 292
    assert q.act_row_bytes(q.Q8_0, 6144) == 192 * 34
    assert q.act_row_bytes(q.F32, 48) == 192
    assert q.act_row_bytes(q.Q4_K, 100) == 0


def test_tune_gemv_ranges_checked_without_gpu(q):
    """qdec_tune_gemv validates every knob on the host: the tile GEMV configuration (0..8), the prefill GEMM's
    column threshold (>= 0) and the warp-MMA GEMV's column threshold (0..4); an unknown kernel is refused."""
    for impl, cfg in ((7, 9), (7, -1), (9, -1), (10, 5), (10, -1), (3, 0), (11, 0)):
        with pytest.raises(q.QdecError) as e:
            q.tune_gemv(impl, cfg)
        assert e.value.code == q.EINVAL
    try:
        for n in (0, 1, 4):
            q.tune_gemv(10, n)
        q.tune_gemv(7, 0)
    finally:
        q.tune_gemv(10, q.GEMV_MMA_MIN_COLS)
        q.tune_gemv(0, 0)
