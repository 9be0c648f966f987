"""The C ABI library: it loads, exports every symbol include/drama3_b200.h declares, and rejects bad arguments
before launching anything. CPU only (no compute call reaches a GPU)."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "drama3_b200.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(d3_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from drama3_b200 import _lib
    return _lib.lib()


def test_library_exports_every_declared_symbol(lib):
    names = declared()
    assert len(names) >= 17
    for name in names:
        assert hasattr(lib, name), name


def test_python_binding_covers_the_header():
    from drama3_b200 import _lib
    assert set(declared()) == set(_lib.SIGNATURES)


def test_version_and_errors(lib):
    assert lib.d3_version() == 100
    assert lib.d3_error_string(0) == b"ok"
    assert b"argument" in lib.d3_error_string(1)


def test_argument_checks_return_before_launch(lib):
    # each of these is rejected on the host (no CUDA call is made)
    assert lib.d3_route(None, 1, 128, 8, None, None, None) == 1
    assert lib.d3_route(1, 1, 2048, 8, 1, 1, None) == 1          # n > 1024
    assert lib.d3_route(1, 1, 128, 33, 1, 1, None) == 1          # k > 32
    assert lib.d3_rotate(1, 0, 1, 100, 1, None, None) == 1       # K % 256
    assert lib.d3_weighted_sum(None, None, 1, 8, 2048, None, None) == 1
    assert lib.d3_moe_decode(0, 16, 1, 17, 8, 128, 2048, 768, *([16] * 12), 1 << 30, None) == 1  # M > 16
    assert lib.d3_moe_decode(9, 16, 1, 1, 8, 128, 2048, 768, *([16] * 12), 1 << 30, None) == 1   # format
    assert lib.d3_moe_decode(0, 16, 1, 1, 8, 128, 2048, 700, *([16] * 12), 1 << 30, None) == 1   # I % 128
    assert lib.d3_moe_decode(0, 16, 1, 4, 8, 128, 2048, 768, *([16] * 12), 16, None) == 5        # workspace
    assert lib.d3_moe_decode(0, 17, 1, 1, 8, 128, 2048, 768, *([16] * 12), 1 << 30, None) == 2   # alignment
    # a1 [M*k, I] + parts [M*k, 2048] fp32, each 256-aligned, + 4096 bytes of synchronization words
    assert lib.d3_moe_decode_workspace(16, 8, 768) == 16 * 8 * (768 + 2048) * 4 + 4096


def test_product_does_not_import_the_oracle():
    pkg = ROOT / "comfyui-drama3_b200"
    for path in pkg.rglob("*.py"):
        text = path.read_text()
        assert "oracle" not in re.sub(r"#.*", "", text).replace('"""', ""), path
