"""CPU checks of the C-ABI boundary: the library loads and exports every declared symbol."""

from __future__ import annotations

import re
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def declared_symbols() -> set[str]:
    names = set()
    for header in (REPO / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"B2P_API\s+[\w\s\*]+?\b(b2p_\w+)\s*\(", text))
    return names


def test_header_declares_every_kernel_entry_point():
    names = declared_symbols()
    for required in ("b2p_kv_write", "b2p_paged_decode", "b2p_paged_prefill",
                     "b2p_build_metadata", "b2p_paged_decode_workspace_size"):
        assert required in names


def test_library_loads_and_exports_all_declared_symbols():
    from llm_engineering_b200 import _lib

    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(_lib.EXPORTED_SYMBOLS) == declared_symbols()
    assert lib.b2p_version() >= 100
    assert _lib.status_text(-2) == "unsupported shape or dtype"


def test_argument_errors_need_no_gpu():
    """Rejections happen on the host before any CUDA call."""
    from llm_engineering_b200 import _lib

    lib = _lib.load()
    # layer index outside the pool
    rc = lib.b2p_kv_write(None, 0, 0, None, 0, 0, None, None, None, 1, 5, 2, 16, 2, 64, 0, None,
                          None)
    assert rc == _lib.B2P_ERANGE
    # q heads not a multiple of kv heads
    rc = lib.b2p_paged_decode(None, 0, 0, None, None, 0, 1, 16, None, 0, None, 1, 7, 2, 64, 16,
                              1.0, None, 0, 0, None, 0, 0, None, None)
    assert rc == _lib.B2P_EINVAL
    assert lib.b2p_paged_decode_workspace_size(256, 12, 2, 128) > 0


def test_lm_head_argmax_rejections_need_no_gpu():
    """K6's argument, shape and workspace checks answer before any CUDA call."""
    from llm_engineering_b200 import _lib

    lib = _lib.load()
    assert lib.b2p_lm_head_argmax_workspace_size(256) == 256 * 8 + 16
    fake = 1 << 20  # an aligned non-null address; nothing is dereferenced on these paths
    # nothing to do
    assert lib.b2p_lm_head_argmax(None, 0, None, 0, 0, 1000, 128, 0, fake, None, None, 0,
                                  None, None) == _lib.B2P_OK
    # negative rows / missing pointers
    assert lib.b2p_lm_head_argmax(fake, 128, fake, 128, -1, 1000, 128, 0, fake, None, fake,
                                  4096, None, None) == _lib.B2P_EINVAL
    assert lib.b2p_lm_head_argmax(None, 128, fake, 128, 128, 1000, 128, 0, fake, None, fake,
                                  4096, None, None) == _lib.B2P_EINVAL
    # fp32, hidden size not a multiple of 64, rows not in 128-row tiles
    for dtype, hidden, rows in ((2, 128, 128), (0, 100, 128), (0, 128, 100)):
        assert lib.b2p_lm_head_argmax(fake, hidden, fake, hidden, rows, 1000, hidden, dtype,
                                      fake, None, fake, 1 << 16, None,
                                      None) == _lib.B2P_EUNSUPPORTED
    # workspace smaller than the rows need
    assert lib.b2p_lm_head_argmax(fake, 128, fake, 128, 256, 1000, 128, 0, fake, None, fake,
                                  256 * 8, None, None) == _lib.B2P_EWORKSPACE
