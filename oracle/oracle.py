"""CPU oracle for the ecq rANS decode + dequant + GEMV path (TEST USE ONLY).

This module is the checker the CUDA path is compared against. Only tests/,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it; the
shipped package (``ecq_b200``) never does.

It wraps ``rans_oracle.c`` (a C restatement of the reference codec, built by
``oracle/Makefile`` into ``oracle/_build/liboracle.so``) and adds numpy code
for the dequant + matvec. Each function names the reference lines it follows
(paths inside drxddy/ecq):

* ``table_reference``    src/rans.py:39-60    (RANSTable.from_counts)
* ``encode_interleaved`` src/interleaved_rans.py:76-153
* ``decode_interleaved`` src/interleaved_rans.py:156-217
* ``dequant_gemv``       src/quantizer.py:33-35 (idx*scale + zero, zero=-8*scale)
                         followed by an fp32/fp64 matvec

Parity of the restatement is pinned against golden vectors made by the
reference's own Python codec (tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

PROB_BITS = 14
PROB_SCALE = 1 << PROB_BITS
RANS_BYTE_L = 1 << 23

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None


def build() -> Path:
    """Compile rans_oracle.c with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < (_HERE / "rans_oracle.c").stat().st_mtime:
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        P = ctypes.c_void_p
        L.oracle_table_reference.argtypes = [P, ctypes.c_int, P]
        L.oracle_table_reference.restype = ctypes.c_int
        L.oracle_table_clamped.argtypes = [P, ctypes.c_int, P]
        L.oracle_table_clamped.restype = None
        L.oracle_table_derive.argtypes = [P, ctypes.c_int, P, P]
        L.oracle_table_derive.restype = None
        L.oracle_encode_interleaved.argtypes = [P, ctypes.c_long, ctypes.c_int, P, P, P]
        L.oracle_encode_interleaved.restype = ctypes.c_long
        L.oracle_decode_interleaved.argtypes = [P, P, ctypes.c_int, ctypes.c_long, P, P, P, P]
        L.oracle_decode_interleaved.restype = ctypes.c_int
        L.oracle_dequant_gemv.argtypes = [P, ctypes.c_long, ctypes.c_long, P, ctypes.c_long, P, P]
        L.oracle_dequant_gemv.restype = None
        L.oracle_gemv_packed.argtypes = [P, P, P, ctypes.c_long, ctypes.c_long, ctypes.c_long, ctypes.c_long,
                                         P, P, ctypes.c_long, P, ctypes.c_long, ctypes.c_long, P]
        L.oracle_gemv_packed.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def table_reference(counts) -> tuple[np.ndarray, int]:
    """Reference normaliser. Returns (freq uint32[16], n_hazard) where
    n_hazard counts present symbols that were given freq 0."""
    c = np.ascontiguousarray(np.asarray(counts, dtype=np.uint64))
    f = np.zeros(len(c), dtype=np.uint32)
    bad = lib().oracle_table_reference(_p(c), len(c), _p(f))
    return f, int(bad)


def table_clamped(counts) -> np.ndarray:
    c = np.ascontiguousarray(np.asarray(counts, dtype=np.uint64))
    f = np.zeros(len(c), dtype=np.uint32)
    lib().oracle_table_clamped(_p(c), len(c), _p(f))
    return f


def table_for(counts) -> tuple[np.ndarray, str]:
    """The reference table unless it has the zero-frequency hazard, in which
    case the clamped table. Returns (freq, normaliser name)."""
    f, bad = table_reference(counts)
    if bad:
        return table_clamped(counts), "clamped"
    return f, "reference"


def table_derive(freq) -> tuple[np.ndarray, np.ndarray]:
    f = np.ascontiguousarray(np.asarray(freq, dtype=np.uint32))
    cum = np.zeros(len(f) + 1, dtype=np.uint32)
    st = np.zeros(PROB_SCALE, dtype=np.uint8)
    lib().oracle_table_derive(_p(f), len(f), _p(cum), _p(st))
    return cum, st


def encode_interleaved(symbols, freq, n_streams: int):
    """Returns (data uint8[S*max_len], stream_lengths uint32[S], max_len)."""
    sym = np.ascontiguousarray(np.asarray(symbols, dtype=np.uint8).reshape(-1))
    f = np.ascontiguousarray(np.asarray(freq, dtype=np.uint32))
    n = sym.size
    S = int(n_streams)
    per = (n + S - 1) // S
    data = np.zeros(S * (2 * per + 8) + 1, dtype=np.uint8)
    lens = np.zeros(S, dtype=np.uint32)
    ml = lib().oracle_encode_interleaved(_p(sym), n, S, _p(f), _p(data), _p(lens))
    if ml == -1:
        raise ValueError("a symbol present in the input has frequency 0")
    if ml < 0:
        raise RuntimeError(f"oracle encode failed ({ml})")
    return data[: S * ml].copy(), lens, int(ml)


def decode_interleaved(data, stream_lengths, n_streams: int, n_symbols: int, freq):
    """Returns (symbols uint8[n], n_bad_streams, end_state[S], end_ptr[S])."""
    d = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8) if isinstance(data, (bytes, bytearray)) else np.asarray(data, dtype=np.uint8))
    S = int(n_streams)
    lens = np.ascontiguousarray(np.asarray(stream_lengths, dtype=np.uint32))
    f = np.ascontiguousarray(np.asarray(freq, dtype=np.uint32))
    out = np.zeros(max(int(n_symbols), 1), dtype=np.uint8)
    es = np.zeros(S, dtype=np.uint32)
    ep = np.zeros(S, dtype=np.uint32)
    # keep a zero tail so a corrupt length never reads past the buffer
    need = S * (int(lens.max()) if S else 0)
    if d.size < need:
        d = np.concatenate([d, np.zeros(need - d.size, dtype=np.uint8)])
    bad = lib().oracle_decode_interleaved(_p(d), _p(lens), S, int(n_symbols), _p(f), _p(out), _p(es), _p(ep))
    return out[: int(n_symbols)], int(bad), es, ep


def dequant_gemv(symbols, scales, group_size: int, x) -> np.ndarray:
    """y[b, r] = sum_c (sym[r,c] - 8) * scale[r, c//g] * x[b, c] in float64,
    returned as float32. symbols uint8 [M,K]; scales [M, ceil(K/g)]; x [B,K]
    or [K]."""
    sym = np.asarray(symbols, dtype=np.uint8)
    M, K = sym.shape
    sc = np.asarray(scales, dtype=np.float64)
    xs = np.asarray(x, dtype=np.float64)
    squeeze = xs.ndim == 1
    xs = xs.reshape(-1, K)
    w = (sym.astype(np.float64) - 8.0) * np.repeat(sc, group_size, axis=1)[:, :K]
    y = xs @ w.T
    y = y.astype(np.float32)
    return y[0] if squeeze else y


def dequant_gemv_c(symbols, scales, group_size: int, x) -> np.ndarray:
    """Same as dequant_gemv for one vector, through the C restatement."""
    sym = np.ascontiguousarray(np.asarray(symbols, dtype=np.uint8))
    M, K = sym.shape
    sc = np.ascontiguousarray(np.asarray(scales, dtype=np.float32))
    xv = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1))
    y = np.zeros(M, dtype=np.float32)
    lib().oracle_dequant_gemv(_p(sym), M, K, _p(sc), int(group_size), _p(xv), _p(y))
    return y


def tile_grid(M: int, K: int, tile_rows: int, tile_cols: int):
    """Tiles of a row-major [M,K] matrix in the order the packed format
    stores them: row-slab major, then K. Yields (row0, rows, col0, cols)."""
    for r0 in range(0, M, tile_rows):
        for c0 in range(0, K, tile_cols):
            yield r0, min(tile_rows, M - r0), c0, min(tile_cols, K - c0)


def encode_matrix_tiles(symbols, freq, tile_rows: int, tile_cols: int, n_streams: int = 32):
    """Encode every tile's row-major symbols with the interleaved codec.
    Returns a list of (data, stream_lengths, max_len) in tile_grid order."""
    sym = np.asarray(symbols, dtype=np.uint8)
    M, K = sym.shape
    out = []
    for r0, nr, c0, nc in tile_grid(M, K, tile_rows, tile_cols):
        out.append(encode_interleaved(sym[r0:r0 + nr, c0:c0 + nc].reshape(-1), freq, n_streams))
    return out


def gemv_packed(data, tile_offset, stream_len, rows, cols, tile_rows, tile_cols, freq, scales, group_size, x,
                threads: int = 1, tile_range=None):
    """The reference CPU path (decode each tile, dequantise, matvec) over a
    packed matrix, using `threads` host threads over disjoint row slabs
    (ctypes releases the GIL). Returns (y float32 [rows], bad_streams)."""
    from concurrent.futures import ThreadPoolExecutor

    d = np.ascontiguousarray(data, dtype=np.uint8)
    off = np.ascontiguousarray(tile_offset, dtype=np.uint32)
    lens = np.ascontiguousarray(stream_len, dtype=np.uint16)
    f = np.ascontiguousarray(freq, dtype=np.uint32)
    sc = np.ascontiguousarray(scales, dtype=np.float32)
    xv = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1))
    y = np.zeros(rows, dtype=np.float64)
    nk = cols // tile_cols
    n_tiles = off.size - 1
    lo, hi = (0, n_tiles) if tile_range is None else tile_range
    slab_lo, slab_hi = lo // nk, (hi + nk - 1) // nk
    threads = max(1, int(threads))
    bounds = np.linspace(slab_lo, slab_hi, threads + 1).astype(np.int64)
    L = lib()

    def run(i):
        t0 = max(lo, int(bounds[i]) * nk)
        t1 = min(hi, int(bounds[i + 1]) * nk)
        if t1 <= t0:
            return 0
        return L.oracle_gemv_packed(_p(d), _p(off), _p(lens), rows, cols, tile_rows, tile_cols, _p(f), _p(sc),
                                    int(group_size), _p(xv), t0, t1, _p(y))

    if threads == 1:
        bad = run(0)
    else:
        with ThreadPoolExecutor(threads) as ex:
            bad = sum(ex.map(run, range(threads)))
    return y.astype(np.float32), int(bad)


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1
