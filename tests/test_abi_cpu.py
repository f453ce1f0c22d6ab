"""CPU-only checks of the boundary: the C ABI library loads and exports every declared symbol, host
argument checking and error reporting work without a GPU, the drop-in Python module keeps the
reference's names and conventions, and the benchmark's model generator writes the reference's
bytes."""
import ctypes
import hashlib
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import PKG, REPO, golden

HEADER = os.path.join(REPO, "include", "eii.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(eii_[a-z_0-9]+)\s*\(", src)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for n in ("eii_open", "eii_open_memory", "eii_close", "eii_forward", "eii_forward_device", "eii_block",
              "eii_embed", "eii_rmsnorm", "eii_linear", "eii_logits", "eii_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import _eii
    lib = ctypes.CDLL(_eii.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_status_and_errors_without_gpu(tmp_path):
    import _eii
    L = _eii.lib()
    assert L.eii_version() == 100
    h = ctypes.c_void_p()
    rc = L.eii_open(str(tmp_path / "missing.bin").encode(), 0, ctypes.byref(h))
    assert rc == _eii.EII_ERR_IO
    assert b"missing.bin" in L.eii_last_error()
    assert L.eii_open(None, 0, ctypes.byref(h)) == _eii.EII_ERR_ARG
    assert L.eii_forward(None, None, 1, 1, None, None, None, None) == _eii.EII_ERR_ARG
    # decoder entry points: a null decoder is an argument error before any device call
    assert L.eii_decoder_step_device(None, None, None, _eii.VOCAB, None, None) == _eii.EII_ERR_ARG
    assert L.eii_decoder_step_device_async(None, None, None, _eii.VOCAB, None, None) == _eii.EII_ERR_ARG
    assert b"decoder is null" in L.eii_last_error()
    assert L.eii_decoder_sync(None, None) == _eii.EII_ERR_ARG
    assert L.eii_decoder_position(None) == -1
    assert L.eii_kernel_name(2) == b"gemm_qkv_rope"


def test_open_without_device_reports_cuda_error(tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import _eii
    with pytest.raises(_eii.EiiError) as ei:
        _eii.Engine(np.zeros(16, np.uint8), 0)
    assert ei.value.code == _eii.EII_ERR_CUDA


def test_cli_usage_and_io_errors(tmp_path):
    cli = os.path.join(PKG, "eii_check")
    if not os.path.exists(cli):
        pytest.skip("eii_check not built")
    r = subprocess.run([cli], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr
    r = subprocess.run([cli, str(tmp_path)], capture_output=True, text=True)
    assert r.returncode == 2


def test_dropin_module_conventions():
    import intref as drop
    from oracle import forward as ofw
    x = np.array([-5, -4, -3, -2, -1, 0, 1, 2, 3, 4, 5, 1 << 40, -(1 << 40)], dtype=np.int64)
    for n in (-3, 0, 1, 2, 7):
        assert np.array_equal(drop.rs(x, n), ofw.rs(x, n))
    assert np.array_equal(drop.sat(x, 16), ofw.sat(x, 16))
    with pytest.raises(AssertionError):
        drop.rs(x, np.zeros_like(x))
    saved = os.environ.pop("EII_MODEL_BIN", None)
    try:
        with pytest.raises(ValueError):
            drop.Model(model_bin=None)
    finally:
        if saved is not None:
            os.environ["EII_MODEL_BIN"] = saved
    assert (drop.F_RES, drop.F_SCORE, drop.DMAX, drop.EPS_S) == (15, 7, 1536, 6184753)


def test_host_digest_matches_definition():
    import _eii
    rng = np.random.default_rng(3)
    lg = rng.integers(-(1 << 31), 1 << 31, size=(2, 3, 49152), dtype=np.int64).astype(np.int32)
    got = _eii.digest_logits(lg)

    def mix(z):
        M = (1 << 64) - 1
        z = (z + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return (z ^ (z >> 31)) | 1
    cols = np.arange(0, 49152, 4099)
    for s in range(2):
        # the definition evaluated with Python ints on a strided sample of columns
        want = sum(int(np.uint32(lg[s, t, v])) * mix(t) * mix((1 << 32) + int(v)) for t in range(3) for v in cols) % (1 << 64)
        sub = np.zeros_like(lg[s:s + 1])
        sub[0][:, cols] = lg[s][:, cols]
        assert int(_eii.digest_logits(sub)[0]) == want
    assert got.dtype == np.uint64
    # one changed logit changes the digest
    lg2 = lg.copy()
    lg2[1, 2, 777] += 1
    assert _eii.digest_logits(lg2)[1] != got[1] and _eii.digest_logits(lg2)[0] == got[0]


def test_package_model_writer_matches_reference_export(tmp_path):
    """bench.py's input generator writes the same bytes as the reference exporter."""
    import synthetic
    p = str(tmp_path / "model.bin")
    synthetic.write_model_bin(p)
    h = hashlib.sha256(open(p, "rb").read()).hexdigest()
    assert h == golden("vectors_t24.json")["files"]["model.bin"]["sha256"]


def test_dropin_formats_follow_fmt(base_model_path):
    """The drop-in builds the engine's format table from Model.fmt (python/intref.py:154-160) over
    the reference's proposal: wide mode reproduces the model.bin's own formats; narrow mode
    (wide=False) gives the narrow table of the reference's formats, with INT16 SiLU tables where
    silu_gate was INT32 (layers 11 and 28); a subclass fmt override (python/ablate_narrow.py:30-40)
    changes exactly the sites it names."""
    import json
    import intref as drop
    fmts = json.load(open(os.path.join(REPO, "oracle", "formats.json")))
    M = drop.Model.__new__(drop.Model)
    M._load(base_model_path, None, wide=True)
    fm, f_y = M._format_table()
    assert [list(r) for r in fm] == fmts["wide"] == M._fm_bin and f_y == fmts["f_y"]
    assert M._model_bin(M._format_table()) == M._base
    M.wide = False
    fm, _ = M._format_table()
    assert [list(r) for r in fm] == fmts["narrow"]
    nb = M._model_bin(M._format_table())
    silu = lambda buf, l: np.frombuffer(buf, np.int64, 65536, M._silu_off[l])
    changed = [l for l in range(30) if not np.array_equal(silu(nb, l), silu(M._base, l))]
    assert changed == [11, 28]
    for l in changed:
        assert silu(nb, l).min() >= -32768 and silu(nb, l).max() <= 32767

    class GatedOnly(drop.Model):  # only the mlp_gated flagged sites narrow (ablate_narrow.py variant)
        def fmt(self, site, l):
            e = self.prop[f"{site}|{l}"]
            if e["class"].startswith("flagged") and (self.wide or site != "mlp_gated"):
                return 32, 31 - e["k"]
            return 16, 15 - e["k"]
    G = GatedOnly.__new__(GatedOnly)
    G._load(base_model_path, None, wide=False)
    gm, _ = G._format_table()
    mi = 2 * 11  # mlp_gated is the 12th site
    for l in range(30):
        for i in range(0, 24, 2):
            want = fmts["narrow"][l] if i == mi else fmts["wide"][l]
            assert list(gm[l][i:i + 2]) == want[i:i + 2], (l, i)
