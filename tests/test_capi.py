"""The C-ABI library loads and exports every function include/ecq.h declares
(no device calls)."""
import re
from pathlib import Path

from ecq_b200 import _lib

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"^\s*(?:int32_t|int64_t|void)\s+(ecq_\w+)\s*\(", text, flags=re.M))
    return sorted(names)


def test_header_and_binding_agree():
    assert declared_functions() == sorted(_lib.EXPORTS)


def test_library_exports_all_symbols():
    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert L.ecq_version() == 100


def test_workspace_size_query_is_host_only():
    v = _lib.MatrixView(rows=4096, cols=4096, tile_rows=8, tile_cols=512, group_size=128, n_tiles=4096)
    assert _lib.lib().ecq_gemv_workspace_bytes(v, 1) == 4096 * 8 * 4 + 512 * 4


def test_tp_comm_struct_mirrors_header():
    import ctypes

    assert ctypes.sizeof(_lib.TPComm) == 4 * 4 + 8 + 8 * _lib.TP_MAX_RANKS
    assert _lib.TPComm.local.offset == 16 and _lib.TPComm.peers.offset == 24
    assert _lib.lib().ecq_comm_buffer_bytes(4096, 8) == 256 + 2 * 8 * 4096 * 8  # (value, epoch) words
    assert _lib.lib().ecq_comm_buffer_bytes(4096, 9) < 0  # more ranks than the exchange holds
