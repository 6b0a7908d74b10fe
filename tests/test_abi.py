"""The C ABI on CPU: the library loads, exports every symbol the header
declares, and fails loudly (an error status, not a fault or a fallback)
where no B200 is present."""

import ctypes as C
import pathlib
import re

import pytest

import emeans_b200
from tests.conftest import has_gpu

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "emeans_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(eb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_device_contract():
    names = declared_functions()
    for want in ["eb_top1", "eb_topk", "eb_scatter_add", "eb_row_norms", "eb_normalize_rows",
                 "eb_split", "eb_ema_update", "eb_bind", "eb_buf_read", "eb_buf_write",
                 "eb_assign", "eb_train", "eb_bind_data", "eb_unbind_data"]:
        assert want in names


def test_library_exports_every_declared_symbol():
    lib = emeans_b200.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_string():
    assert b"sm_100a" in emeans_b200.load().eb_version()


@pytest.mark.skipif(has_gpu(), reason="checks the no-device error path")
def test_engine_without_device_is_an_error_not_a_fallback():
    with pytest.raises(emeans_b200.EngineError) as ei:
        emeans_b200.Engine(0)
    assert ei.value.code == emeans_b200.ERROR


def test_null_arguments_are_invalid():
    lib = emeans_b200.load()
    assert lib.eb_sync(None) == emeans_b200.INVALID_ARGUMENT
    assert b"null" in lib.eb_last_error()
    out = C.c_void_p()
    assert lib.eb_buf_alloc(None, 0, 4, C.byref(out)) == emeans_b200.INVALID_ARGUMENT
    assert lib.eb_train(None, None, None) == emeans_b200.INVALID_ARGUMENT


def test_load_fails_loudly_when_library_missing(monkeypatch, tmp_path):
    monkeypatch.setattr(emeans_b200, "_lib", None)
    monkeypatch.setattr(emeans_b200, "HERE", str(tmp_path))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        emeans_b200.load()


def test_view_outside_its_buffer_is_refused():
    """Engine.view checks its range before any C call: a view past the
    buffer's end, or a negative one, is INVALID_ARGUMENT."""

    class FakeBuffer:
        ptr = 4096

        def __len__(self):
            return 64

    for offset, length in [(60, 8), (-4, 4), (0, 65), (8, -1)]:
        with pytest.raises(emeans_b200.EngineError) as err:
            emeans_b200.Engine.view(None, FakeBuffer(), offset, length, emeans_b200.U32)
        assert err.value.code == emeans_b200.INVALID_ARGUMENT
