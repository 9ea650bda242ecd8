"""libecq's C ABI driven from a plain C program (tests/c/abi_host_example.c,
compiled here with the system C compiler): the table normaliser, the
interleaved host encoder and the decode-table builder, checked against the
oracle. Host functions only, no GPU."""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from ecq_b200 import _lib
from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]


def _symbols(n):
    x, out = 12345, np.empty(n, dtype=np.uint8)
    for i in range(n):
        x = (x * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        u = (x >> 40) % 1000
        out[i] = 8 if u < 600 else 7 if u < 760 else 9 if u < 920 else 6 if u < 950 else 10 if u < 980 else \
            (5 if u & 1 else 11)
    return out


@pytest.mark.parametrize("n", [1, 33, 4099])
def test_c_program_through_the_abi(tmp_path, n):
    cc = shutil.which("cc") or shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    libdir = Path(_lib.lib()._name).parent
    exe = tmp_path / "example"
    subprocess.run([cc, "-O2", "-I", str(ROOT / "include"), str(ROOT / "tests" / "c" / "abi_host_example.c"),
                    f"-L{libdir}", "-lecq", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe), str(n)], check=True, capture_output=True, text=True).stdout
    f = dict(line.split(" ", 1) for line in out.strip().splitlines())
    sym = _symbols(n)
    freq = np.array(f["freq"].split(), dtype=np.uint32)
    assert freq.sum() == 16384
    ref_freq, ref_norm = oracle.table_for(np.bincount(sym, minlength=16))
    assert np.array_equal(freq, ref_freq)
    assert int(f["normaliser"]) == (0 if ref_norm == "reference" else 1)
    data = bytes.fromhex(f["data"].strip())
    lens = [int(v) for v in f["lens"].split()]
    ref_data, ref_lens, ref_max = oracle.encode_interleaved(sym, freq, 32)
    assert data == bytes(ref_data) and lens == list(ref_lens) and int(f["max_len"]) == ref_max
    dec, bad, _, _ = oracle.decode_interleaved(data, np.array(lens, np.uint32), 32, n, freq)
    assert bad == 0 and np.array_equal(dec, sym)
    # every slot's entry: (slot - cumfreq[s]) | s << 14 | freq[s] << 18
    f64 = freq.astype(np.int64)
    cum = np.concatenate([[0], np.cumsum(f64)])
    s_of = np.repeat(np.arange(16, dtype=np.int64), f64)
    entries = (np.arange(16384, dtype=np.int64) - cum[s_of]) | (s_of << 14) | (f64[s_of] << 18)
    assert int(f["table_sum"]) == int(entries.sum())
