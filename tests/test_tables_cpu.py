"""Independent regeneration of the model.bin tables (python/intref.py:66-108) by the engine library,
on the CPU (no device): pinned to digests of the reference's own mpmath tables (tests/golden/tables.json,
written by make_golden.py --only-tables), and cross-checked against every table of the
reference-identical synthetic model.bin files."""
import time

import numpy as np
import pytest

from conftest import golden, sha256_arr


def test_exp_and_rope_tables_match_reference_digests():
    import _eii
    g = golden("tables.json")["tables"]
    assert sha256_arr(_eii.table_exp(), np.int64) == g["exp"]
    c, s = _eii.table_rope(512)
    assert sha256_arr(c, np.int64) == g["rope_cos"]
    assert sha256_arr(s, np.int64) == g["rope_sin"]


def test_silu_tables_match_reference_digests():
    """Every (f_g, f_s, bits_s) pair of the reference's format table, wide and narrow."""
    import _eii
    g = golden("tables.json")["tables"]["silu"]
    t0 = time.time()
    for key, want in g.items():
        fi, fo, b = (int(v) for v in key.split(","))
        assert sha256_arr(_eii.table_silu(fi, fo, b), np.int64) == want, key
    assert time.time() - t0 < 60


def test_verify_model_bin_tables(base_model_path, outlier_model_path):
    import _eii
    _eii.verify_tables(base_model_path)
    _eii.verify_tables(outlier_model_path)


@pytest.mark.parametrize("where", ["exp", "rope", "silu"])
def test_verify_tables_detects_one_unit(base_model_path, where):
    """A one-unit change in one table entry is reported with its position."""
    import _eii
    buf = bytearray(open(base_model_path, "rb").read())
    V, D = 49152, 576
    off = V * D + 16 * V + 8 * (D + 1) + 8
    if where == "rope":
        off += 8 * 1537 + 8 * (5 * 32 + 7)
    elif where == "silu":
        off = len(buf) - 8 * 65536 + 8 * 40000
    else:
        off += 8 * 100
    v = int.from_bytes(buf[off:off + 8], "little", signed=True) + 1
    buf[off:off + 8] = v.to_bytes(8, "little", signed=True)
    with pytest.raises(_eii.EiiError) as ei:
        _eii.verify_tables(bytes(buf))
    assert ei.value.code == _eii.EII_ERR_FORMAT
    assert "differs" in str(ei.value)


def test_table_arguments():
    import _eii
    with pytest.raises(_eii.EiiError):
        _eii.table_silu(-1, 8, 16)
    with pytest.raises(_eii.EiiError):
        _eii.table_rope(0)
