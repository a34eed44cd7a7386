"""CPU: the C-ABI library loads, exports every symbol include/s2k.h declares,
and fails cleanly (no crash, a status code) when no GPU is visible."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

import s2k
import synthetic

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols() -> list[str]:
    txt = open(os.path.join(ROOT, "include", "s2k.h")).read()
    return sorted(set(re.findall(r"S2K_API\s+[^;(]*?\b(s2k_\w+)\s*\(", txt, flags=re.S)))


def test_header_and_binding_agree():
    assert header_symbols() == sorted(s2k.EXPORTED)


def test_library_exports_header_symbols():
    L = s2k.lib()
    for name in header_symbols():
        assert hasattr(L, name), name
    assert L.s2k_abi_version() == 1


def test_hparams_struct_layout_matches_header():
    # 29 four-byte fields, in header order
    assert ctypes.sizeof(s2k._HParams) == 29 * 4
    assert [f for f, _ in s2k._HParams._fields_] == synthetic.FIELDS


@pytest.mark.skipif(s2k.device_count() > 0, reason="checks the no-GPU error path")
def test_no_device_error_paths():
    assert s2k.device_count() == 0
    with pytest.raises(s2k.S2KError) as e:
        s2k.SlowARModel(synthetic.preset("small"))
    assert e.value.status == -8
    msg = s2k.lib().s2k_last_error().decode()
    assert msg


def test_sched_stats_struct_layout_matches_header():
    txt = open(os.path.join(ROOT, "include", "s2k.h")).read()
    body = re.search(r"typedef struct \{(.*?)\} s2k_sched_stats;", txt, flags=re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if decl:
            names += [n.strip() for n in decl.split(None, 1)[1].split(",")]
    assert names == [f for f, _ in s2k._SchedStats._fields_]
    # 6 int64, 4 int32, 2 int64
    assert ctypes.sizeof(s2k._SchedStats) == 80
