"""C ABI checks that need no GPU: the library loads, exports every entry
point the header declares, and the ctypes structs match the C layout."""
import ctypes
import re
import subprocess
import tempfile
from pathlib import Path

import pytest

from infercache_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "infercache.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ic_[a-z_0-9]+)\s*\(", text)))


def test_library_loads():
    lib = _lib.load()
    assert lib.ic_abi_version() == 3


def test_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 16
    for n in names:
        assert hasattr(lib, n), n
    # and the binding covers exactly the declared entry points
    assert set(names) == set(_lib.ENTRY_POINTS) | set(_lib.INFO_ENTRY_POINTS) | set(_lib.HOST_ENTRY_POINTS)


def test_status_strings():
    lib = _lib.load()
    assert lib.ic_status_str(0) == b"ok"
    assert lib.ic_status_str(_lib.IC_ERR_OUT_OF_PAGES) == b"page pool exhausted"
    assert lib.ic_status_str(12345) == b"unknown status"


def test_host_device_pointer_rejects_null_without_cuda_call():
    lib = _lib.load()
    import ctypes
    assert lib.ic_host_device_pointer(None, None) == _lib.IC_ERR_INVALID_ARG
    out = ctypes.c_void_p()
    assert lib.ic_host_device_pointer(None, ctypes.byref(out)) == _lib.IC_ERR_INVALID_ARG


def test_wait_probe_rejects_bad_args_without_cuda_call():
    lib = _lib.load()
    assert lib.ic_wait_probe(None, 1000, None) == _lib.IC_ERR_INVALID_ARG
    import ctypes
    x = ctypes.c_int32(0)
    assert lib.ic_wait_probe(ctypes.addressof(x), 0, None) == _lib.IC_ERR_INVALID_ARG
    assert lib.ic_wait_probe(ctypes.addressof(x), 3_000_000_000, None) == _lib.IC_ERR_INVALID_ARG


def test_null_args_rejected_without_launch():
    """Argument validation runs on the host before any CUDA call."""
    lib = _lib.load()
    for name in _lib.ENTRY_POINTS:
        assert getattr(lib, name)(None, None) == _lib.IC_ERR_INVALID_ARG, name


def test_struct_layout_matches_c():
    structs = {n: st for n, st in _lib.ENTRY_POINTS.items()}
    structs.update({"pool": _lib.ic_pool, "tiers": _lib.ic_tiers, "sess": _lib.ic_sessions})
    cnames = {st.__name__ for st in structs.values()}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cn in sorted(cnames):
        st = getattr(_lib, cn)
        lines.append(f'printf("{cn} %zu\\n", sizeof({cn}));')
        for fname, _ in st._fields_:
            lines.append(f'printf("{cn}.{fname} %zu\\n", offsetof({cn}, {fname}));')
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        src = Path(d) / "layout.c"
        exe = Path(d) / "layout"
        src.write_text("\n".join(lines))
        r = subprocess.run(["gcc", "-std=c99", str(src), "-o", str(exe)], capture_output=True, text=True)
        if r.returncode != 0:
            pytest.fail(r.stderr)
        out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    c = dict(line.split() for line in out.strip().splitlines())
    for cn in sorted(cnames):
        st = getattr(_lib, cn)
        assert int(c[cn]) == ctypes.sizeof(st), cn
        for fname, _ in st._fields_:
            assert int(c[f"{cn}.{fname}"]) == getattr(st, fname).offset, f"{cn}.{fname}"


def test_no_cpu_path():
    """Constructing a cache without an sm_100 device fails loudly."""
    import torch
    from infercache_b200 import CacheConfig, HierarchicalKVCache
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    cfg = CacheConfig(num_layers=1, num_kv_heads=2, head_dim=128)
    with pytest.raises(Exception):
        HierarchicalKVCache(cfg, device="cpu")
    with pytest.raises(Exception):
        HierarchicalKVCache(cfg, device="cuda")
