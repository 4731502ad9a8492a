"""The C-ABI library loads without a GPU and exports every declared symbol.

No compute entry point is called here (there is no device); only the
host-side functions (version, status strings, launch table, workspace size).
"""
import ctypes
import os
import re

import pytest

from dsa_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dsa_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DSA_B200_API\s+[\w\s\*]*?\b(dsa_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_native.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings():
    lib = _native.load()
    assert lib.dsa_abi_version() == _native.ABI_VERSION
    for code in range(7):
        assert _native.status_string(code)
    assert _native.status_string(0) == "ok"


def test_default_launch_is_shape_only_and_valid():
    lib = _native.load()
    for shape in [(1, 1, 128, 4096, 2048), (8, 2, 128, 32768, 2048), (64, 1, 16, 65536, 2048),
                  (1, 4096, 16, 8192, 2048), (4, 4096, 128, 65536, 2048), (1, 3, 32, 100, 77)]:
        a, b = _native.Launch(), _native.Launch()
        assert lib.dsa_default_launch(*shape, ctypes.byref(a)) == 0
        assert lib.dsa_default_launch(*shape, ctypes.byref(b)) == 0
        assert bytes(a) == bytes(b)
        assert lib.dsa_check_launch(*shape, ctypes.byref(a)) == 0
        tiles = -(-shape[4] // a.keys_per_tile)
        assert 1 <= a.split <= tiles


def test_check_launch_rejections():
    lib = _native.load()
    shape = (1, 1, 32, 1024, 256)
    for fam, bm, bn, split in [(1, 16, 48, 1), (1, 32, 32, 1), (1, 16, 32, 0), (1, 16, 32, 9), (7, 16, 32, 1)]:
        e = _native.Launch(fam, bm, bn, split)
        assert lib.dsa_check_launch(*shape, ctypes.byref(e)) != 0, (fam, bm, bn, split)
    assert lib.dsa_check_launch(1, 1, 24, 1024, 256, ctypes.byref(_native.Launch(1, 16, 32, 1))) != 0
    # keys family: 64-key tiles only
    assert lib.dsa_check_launch(*shape, ctypes.byref(_native.Launch(_native.FAMILY_KEYS, 16, 64, 4))) == 0
    assert lib.dsa_check_launch(*shape, ctypes.byref(_native.Launch(_native.FAMILY_KEYS, 16, 32, 1))) != 0
    assert lib.dsa_check_launch(*shape, ctypes.byref(_native.Launch(_native.FAMILY_KEYS, 16, 64, 5))) != 0
    assert lib.dsa_check_launch(0, 1, 32, 1024, 256, ctypes.byref(_native.Launch(1, 16, 32, 1))) != 0


def test_workspace_bytes():
    lib = _native.load()
    args = _native.FwdArgs()
    args.batch, args.queries, args.heads, args.length, args.topk = 2, 3, 32, 1024, 256
    args.launch = _native.Launch(1, 16, 32, 1)
    assert lib.dsa_fwd_workspace_bytes(ctypes.byref(args)) == 0
    args.launch = _native.Launch(1, 16, 32, 4)
    rows = 2 * 3 * 4 * 32
    ws = lib.dsa_fwd_workspace_bytes(ctypes.byref(args))
    assert ws >= rows * 512 * 4 + 2 * rows * 4 and ws % 256 == 0


def test_forward_fails_loudly_without_library(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(RuntimeError, match="no fallback"):
        _native.load()


def test_union_launch_topk_bound():
    """The union launch counts a key's repeats per query in 16 bits: TOPK
    above 65535 is refused for it (and the default never picks it then)."""
    lib = _native.load()
    union = _native.Launch(_native.FAMILY_PAIR_UNION, 128, 32, 1)
    assert lib.dsa_check_launch(1, 8, 16, 1 << 20, 65535, ctypes.byref(union)) == 0
    assert lib.dsa_check_launch(1, 8, 16, 1 << 20, 65536, ctypes.byref(union)) == _native.STATUS_UNSUPPORTED
    e = _native.Launch()
    assert lib.dsa_default_launch(1, 8192, 16, 200000, 65536, ctypes.byref(e)) == 0
    assert e.family != _native.FAMILY_PAIR_UNION


def test_wait_test_hook_is_host_only():
    """The failure-path test hook only sets host-side values for later launches."""
    lib = _native.load()
    assert lib.dsa_set_wait_test(1000, 1) == 0
    assert lib.dsa_set_wait_test(0, 0) == 0
