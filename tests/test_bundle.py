"""The drafter bundle format (MRBDRFT1, drafting/export_drafter.py:12-35): write/read round trip and
interchange with the reference's own writer/reader."""

from __future__ import annotations

import numpy as np
import pytest

from tests.golden import cases


def test_roundtrip_and_alignment(lngram, tmp_path):
    config, arrays = cases.draft_bundle("tiny")
    arrays = dict(arrays, **cases.random_sketch(config))
    path = lngram.write_bundle(tmp_path / "b.bin", config, arrays, {"note": "x"})
    head = lngram.read_header(path)
    assert head["version"] == 1
    for meta in head["arrays"].values():
        assert meta["offset"] % 64 == 0
    for mmap in (True, False):
        b = lngram.load_bundle(path, mmap=mmap)
        assert b.config == config and b.source == {"note": "x"}
        for k, v in arrays.items():
            assert b.arrays[k].dtype == v.dtype
            np.testing.assert_array_equal(b.arrays[k], v)
    with pytest.raises(ValueError):
        (tmp_path / "bad.bin").write_bytes(b"NOTABUNDLE" + b"\0" * 16)
        lngram.read_header(tmp_path / "bad.bin")


@pytest.mark.reference
def test_interchange_with_reference_format(lngram, reference_path, tmp_path):
    from drafting.export_drafter import load_bundle as ref_load
    from drafting.export_drafter import write_bundle as ref_write

    config, arrays = cases.draft_bundle("tiny")
    arrays = dict(arrays, **cases.random_sketch(config))       # uint16 ids / uint32 counts / int32 fallback too
    p1 = ref_write(tmp_path / "ref.bin", config, arrays, {"s": 1})
    ours = lngram.load_bundle(p1)
    p2 = lngram.write_bundle(tmp_path / "ours.bin", config, arrays, {"s": 1})
    theirs = ref_load(p2)
    assert p1.read_bytes() == p2.read_bytes()
    for k in arrays:
        np.testing.assert_array_equal(ours.arrays[k], arrays[k])
        np.testing.assert_array_equal(theirs.arrays[k], arrays[k])
