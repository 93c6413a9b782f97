"""CPU checks of the C ABI: libinferc_b200.so exists, loads, and exports
every function that include/*.h declares; the ctypes table in
inferc_b200/lib.py covers all of them; host-side logic (DP sharding)."""
import glob
import os
import re

import pytest

from inferc_b200 import dp, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols() -> set[str]:
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(inferc_dev_\w+)\s*\(", text))
    return names


def test_library_is_built_in_tree():
    assert os.path.exists(lib.LIB_PATH), "run python -m inferc_b200.build"


def test_library_exports_every_declared_symbol():
    L = lib.load()
    declared = declared_symbols()
    assert len(declared) >= 25
    missing = [n for n in sorted(declared) if not hasattr(L, n)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    assert set(lib.SIGNATURES) == declared_symbols()


def test_version_string_callable_without_gpu():
    assert b"sm_100a" in lib.load().inferc_dev_version()


def test_shard_rows_cover_batch_exactly():
    for total in (0, 1, 7, 256, 257):
        for world in (1, 2, 3, 4, 8):
            spans = [dp.shard_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_shard_rows_rejects_bad_rank():
    with pytest.raises(ValueError):
        dp.shard_rows(8, 2, 2)
