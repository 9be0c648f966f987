"""The library called from plain C through include/drama3_b200.h (tests/c_abi/pack_caller.c, built with gcc and
linked against libdrama3_b200.so): its host packers give the same bytes as the Python binding's, so the C boundary
is usable without Python. CPU only."""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from drama3_b200 import _lib, pack

ROOT = Path(__file__).resolve().parents[1]


def fnv(h, data):
    for b in np.ascontiguousarray(data).view(np.uint8).reshape(-1).tolist():
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def checksum(*arrays):
    h = 14695981039346656037
    for a in arrays:
        h = fnv(h, a)
    return f"{h:016x}"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_c_caller_matches_python(tmp_path):
    lib = _lib.LIB_PATH
    exe = tmp_path / "pack_caller"
    subprocess.run(["gcc", "-std=c99", "-O1", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_abi" / "pack_caller.c"), "-L", str(lib.parent), "-ldrama3_b200",
                    f"-Wl,-rpath,{lib.parent}", "-o", str(exe)], check=True)
    rows_path = tmp_path / "rows.f32"
    run = subprocess.run([str(exe), str(rows_path)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    got = dict(line.split() for line in run.stdout.splitlines())
    w = torch.from_numpy(np.fromfile(rows_path, np.float32).reshape(256, 512))
    want = {}
    for kind in ("fp8", "int8", "w4", "w6", "fp8c", "w4a8", "w6a8"):
        f = pack.pack_bank(kind, w)
        if kind in ("w4a8", "w6a8"):
            want[kind] = checksum(f["_qdata"].numpy(), f["scale"].view(torch.int16).numpy())
        elif kind in ("w4", "w6"):
            want[kind] = checksum(f["_qdata"].numpy(), f["scale"].numpy(), f["s_channel"].numpy())
        else:
            key = "weight" if kind in ("fp8", "fp8c") else "_qdata"
            want[kind] = checksum(f[key].numpy(), f["scale"].numpy())
    assert got == want
