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
    assert set(names) == (set(_lib.ENTRY_POINTS) | set(_lib.BATCH_ENTRY_POINTS) | set(_lib.INFO_ENTRY_POINTS)
                          | set(_lib.HOST_ENTRY_POINTS))
    text = HEADER.read_text()
    assert re.search(rf"#define IC_PAGE_BATCH_MAX {_lib.IC_PAGE_BATCH_MAX}\b", text)


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


def test_graph_replay_rejects_bad_args_without_cuda_call():
    import ctypes
    lib = _lib.load()
    arr = (ctypes.c_void_p * 2)(1, 2)
    nul = (ctypes.c_void_p * 2)(1, None)
    assert lib.ic_graph_replay(None, arr, 2, 1) == _lib.IC_ERR_INVALID_ARG
    assert lib.ic_graph_replay(arr, None, 2, 1) == _lib.IC_ERR_INVALID_ARG
    assert lib.ic_graph_replay(arr, arr, 0, 1) == _lib.IC_ERR_INVALID_ARG
    assert lib.ic_graph_replay(arr, arr, 2, -1) == _lib.IC_ERR_INVALID_ARG
    assert lib.ic_graph_replay(nul, arr, 2, 1) == _lib.IC_ERR_INVALID_ARG
    assert lib.ic_graph_replay(arr, arr, 2, 0) == _lib.IC_OK  # nothing to launch


def test_evict_pdl_mode_checked_without_cuda_call():
    """ic_evict_update accepts pdl 0, 1 or 2 only; the check precedes any CUDA call."""
    import ctypes
    lib = _lib.load()
    buf = (ctypes.c_int64 * 64)()
    p = ctypes.addressof(buf)
    sess = _lib.ic_sessions(num_sessions=1, slot_table=p, positions=p, importance=p, occupied=p, ctrl=p,
                            counters=p)
    for pdl in (-1, 3):
        e = _lib.ic_evict_args(tiers=_lib.ic_tiers(sink_size=1, recent_size=2, important_size=3, budget=6),
                               sess=sess, pdl=pdl, new_pos=p)
        assert lib.ic_evict_update(ctypes.byref(e), None) == _lib.IC_ERR_INVALID_ARG, pdl


def test_null_args_rejected_without_launch():
    """Argument validation runs on the host before any CUDA call."""
    lib = _lib.load()
    for name in _lib.ENTRY_POINTS:
        assert getattr(lib, name)(None, None) == _lib.IC_ERR_INVALID_ARG, name
    for name in _lib.BATCH_ENTRY_POINTS:
        assert getattr(lib, name)(None, 1, None) == _lib.IC_ERR_INVALID_ARG, name


def test_page_batch_checks_without_cuda_call():
    """Batched page gathers: the count bound, one pool and one layer range for
    every descriptor, all checked before any CUDA call."""
    import ctypes
    lib = _lib.load()
    buf = (ctypes.c_int64 * 256)()
    p = ctypes.addressof(buf)
    p = (p + 15) // 16 * 16
    pool = _lib.ic_pool(k=p, v=p, pool_tokens=64, num_layers=2, num_kv_heads=1, head_dim=128, dtype=1)

    def desc(**kw):
        d = dict(pool=pool, page_ids=p, n_page_ids=2, layer_begin=0, layer_end=2, start_token=0, n_tokens=8,
                 k_buf=p, v_buf=p, stride_l=128 * 8, stride_h=128 * 8, stride_t=128)
        d.update(kw)
        return _lib.ic_page_rows_args(**d)

    for name in _lib.BATCH_ENTRY_POINTS:
        fn = getattr(lib, name)
        arr = (_lib.ic_page_rows_args * (_lib.IC_PAGE_BATCH_MAX + 1))(*[desc() for _ in range(_lib.IC_PAGE_BATCH_MAX + 1)])
        assert fn(arr, 0, None) == _lib.IC_ERR_INVALID_ARG
        assert fn(arr, _lib.IC_PAGE_BATCH_MAX + 1, None) == _lib.IC_ERR_INVALID_ARG
        other = _lib.ic_pool(k=p + 16, v=p, pool_tokens=64, num_layers=2, num_kv_heads=1, head_dim=128, dtype=1)
        for bad in (desc(pool=other), desc(layer_end=1), desc(n_tokens=-1), desc(n_tokens=40),
                    desc(stride_t=100)):
            two = (_lib.ic_page_rows_args * 2)(desc(), bad)
            assert fn(two, 2, None) == _lib.IC_ERR_INVALID_ARG, name


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
