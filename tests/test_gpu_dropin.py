"""The drop-in Python module (exact-integer-inference_b200/intref.py) under the reference's own callers.

* python/export_vectors.py:14-58, replayed call for call through the drop-in (Model, M.prop, M.fmt,
  M.rope, silu_table, exp_table, embed, block, rmsnorm, matmul_exact, rs): the model.bin and the
  exported states must have the sha256 of the reference's own export (tests/golden/vectors_t24.json).
* The conformance checker (eii_check) on that vector set, and the reference's negative test
  (tools/record_conformance.sh:44-62: one unit added to the middle int32 of exp_resid_out.i32).
* Model subclasses with the fmt and _grid overrides of the reference's ablation scripts against
  the reference's own logits (tests/golden/ablation_t24.json).
* rmsnorm(trace=...) and matmul_exact with a non-int8 right operand."""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import GOLDEN, PKG, golden, sha256_arr, sha256_file
from oracle import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def drop():
    import intref
    return intref


def _export(drop, M, outdir, ids):
    """python/export_vectors.py:14-58 through the drop-in module."""
    os.makedirs(outdir, exist_ok=True)

    def w(f, a, dt):
        f.write(np.ascontiguousarray(a, dtype=dt).tobytes())
    with open(os.path.join(outdir, "model.bin"), "wb") as f:
        w(f, M.emb_q, np.int8); w(f, M.emb_m, np.int64); w(f, M.emb_n, np.int64)
        w(f, M.final_gain[0], np.int64); w(f, [M.final_gain[1]], np.int64)
        w(f, [15 - M.prop["final_out|30"]["k"]], np.int64)
        w(f, drop.exp_table(), np.int64)
        C, S = M.rope
        w(f, C[:512], np.int64); w(f, S[:512], np.int64)
        names = ["norm1_out", "q_proj", "k_proj", "v_proj", "q_rope", "k_rope", "attn_ctx", "norm2_out", "gate_proj",
                 "up_proj", "silu_gate", "mlp_gated"]
        for l in range(M.L):
            Ly = M.layers[l]
            fm = []
            for nme in names:
                bits, fr = M.fmt(nme, l)
                fm += [bits, fr]
            w(f, fm, np.int64)
            w(f, Ly["ln1"][0], np.int64); w(f, [Ly["ln1"][1]], np.int64)
            w(f, Ly["ln2"][0], np.int64); w(f, [Ly["ln2"][1]], np.int64)
            for nme in ("q", "k", "v", "o", "gate", "up", "down"):
                q, m, n = Ly[nme]
                w(f, q, np.int8); w(f, m, np.int64); w(f, n, np.int64)
            _, f_g = M.fmt("gate_proj", l)
            bits_s, f_s = M.fmt("silu_gate", l)
            w(f, drop.silu_table(f_g, f_s, bits_s), np.int64)
    x = M.embed(ids)
    exp_embed = x.copy()
    res = []
    for l in range(M.L):
        x = M.block(l, x)
        res.append(x.copy())
    bits_y, f_y = 16, 15 - M.prop["final_out|30"]["k"]
    y = M.rmsnorm(x, M.final_gain, f_y, bits_y)
    acc = drop.matmul_exact(y, M.emb_q, 1 << 15)
    logits = drop.rs(acc * M.emb_m[None, :], M.emb_n + f_y - 16)
    assert np.abs(logits).max() < 2 ** 31 and np.abs(np.array(res)).max() < 2 ** 31
    for name, arr, dt in (("ids.i64", ids, np.int64), ("exp_embed.i32", exp_embed, np.int32),
                          ("exp_resid_out.i32", np.array(res), np.int32), ("exp_logits.i32", logits, np.int32)):
        np.ascontiguousarray(arr, dtype=dt).tofile(os.path.join(outdir, name))
    return logits


def test_export_vectors_replay_matches_reference_export(drop, base_model_path, tmp_path):
    g = golden("vectors_t24.json")
    M = drop.Model(model_bin=base_model_path)
    try:
        ids = synth.window_ids(g["window"], g["tokens"])
        d = str(tmp_path / "t24")
        logits = _export(drop, M, d, ids)
        for fn, want in g["files"].items():
            assert sha256_file(os.path.join(d, fn)) == want["sha256"], fn
        # Model.forward: one engine call, int64 logits
        assert np.array_equal(M.forward(ids), logits)
        # the conformance checker on the exported set, then the reference's negative test
        cli = os.path.join(PKG, "eii_check")
        r = subprocess.run([cli, d], capture_output=True, text=True)
        assert r.returncode == 0 and "ALL STATES EXACT" in r.stdout, r.stdout + r.stderr
        assert r.stdout.count(": exact") == 31  # 30 layers and the logits
        bad = str(tmp_path / "t24_bad")
        os.makedirs(bad)
        for fn in os.listdir(d):
            if fn != "model.bin":
                with open(os.path.join(d, fn), "rb") as src, open(os.path.join(bad, fn), "wb") as dst:
                    dst.write(src.read())
        p = os.path.join(bad, "exp_resid_out.i32")
        b = bytearray(open(p, "rb").read())
        i = len(b) // 2 // 4 * 4
        b[i:i + 4] = (int.from_bytes(b[i:i + 4], "little", signed=True) + 1).to_bytes(4, "little", signed=True)
        open(p, "wb").write(b)
        r = subprocess.run([cli, bad, d], capture_output=True, text=True)
        assert r.returncode == 1, r.stdout + r.stderr
        assert "DIFFERS" in r.stdout and "MISMATCH" in r.stdout and "FAIL" in r.stdout
    finally:
        M.close()


def _ablation_shifts():
    sys.path.insert(0, GOLDEN)
    from make_golden import ablation_shifts
    return ablation_shifts()


@pytest.mark.parametrize("variant", ["flagged_gated_only", "flagged_ctx_silu_only", "channel_grid",
                                     "channel_grid_on_gpu", "grid_layers_12_28"])
def test_subclass_overrides_match_reference(drop, base_model_path, variant):
    """fmt and _grid overrides of the reference's ablation scripts, through the drop-in module."""
    g = golden("ablation_t24.json")
    want = g["variants"][variant.replace("_on_gpu", "")]
    ids = synth.window_ids(g["window"], g["tokens"])

    class NarrowSites(drop.Model):
        narrow_sites = None

        def fmt(self, site, l):
            e = self.prop[f"{site}|{l}"]
            if e["class"].startswith("flagged"):
                if self.wide or (self.narrow_sites is not None and site not in self.narrow_sites):
                    return 32, 31 - e["k"]
            return 16, 15 - e["k"]

    pcs = _ablation_shifts()

    class ChannelGrid(drop.Model):  # the reference's form: its own _grid, applied on the host
        def _grid(self, x, site, l):
            s = pcs[(site, l)][None, :]
            half = np.where(s > 0, np.int64(1) << np.maximum(s - 1, 0), 0)
            y = np.where(s > 0, (x + half) >> s, x)
            return drop.sat(y, 16) << s

    class ChannelGridOnGpu(drop.Model):  # the same grid as per-channel shifts, applied on the GPU
        def grid_shifts(self, site, l):
            return pcs[(site, l)]

    class SomeLayers(drop.Model):
        def _grid(self, x, site, l):
            return super()._grid(x, site, l) if 12 <= l < 29 else x

    if variant.startswith("flagged"):
        M = NarrowSites(wide=False, model_bin=base_model_path)
        M.narrow_sites = {"mlp_gated"} if variant == "flagged_gated_only" else {"attn_ctx", "silu_gate"}
        nres = False
    else:
        cls = {"channel_grid": ChannelGrid, "channel_grid_on_gpu": ChannelGridOnGpu, "grid_layers_12_28": SomeLayers}[variant]
        M = cls(wide=True, model_bin=base_model_path)
        nres = True
    try:
        lg = M.forward(ids, narrow_residual=nres)
    finally:
        M.close()
    assert lg[0, :8].tolist() == want["logits_row0_first8"]
    assert sha256_arr(lg, np.int64) == want["logits_int64_sha256"]


def test_rmsnorm_trace_matches_reference(drop, base_model, base_model_path):
    """Model.rmsnorm(x, gain, f_out, bits_out, trace, tag) fills U, z and out as the reference's
    trace does (its layer-0 norm1 digests, tests/golden/trace_t24.json)."""
    from test_oracle_golden import trace_inputs
    g, xs = trace_inputs(base_model)
    sites = g["layers"]["0"]["sites"]
    M = drop.Model(model_bin=base_model_path)
    try:
        bits_h, f_h = M.fmt("norm1_out", 0)
        tr = {}
        out = M.rmsnorm(xs[0], M.layers[0]["ln1"], f_h, bits_h, trace=tr, tag="norm1")
    finally:
        M.close()
    for k in ("norm1_U", "norm1_z", "norm1_out"):
        assert sha256_arr(tr[k], np.int64) == sites[k]["sha256"], k
    assert np.array_equal(out, tr["norm1_out"])


def test_matmul_exact_wide_right_operand(drop, base_model_path):
    """matmul_exact with INT16 and wider right operands (python/intref.py:238 multiplies q by k),
    ragged K and N, against exact int64 products."""
    rng = np.random.default_rng(4)
    M = drop.Model(model_bin=base_model_path)
    try:
        for T, K, N, bound, wb in ((24, 64, 24, 1 << 15, 1 << 15), (7, 100, 33, 1 << 31, 1 << 20), (5, 576, 16, 1 << 15, 127)):
            A = rng.integers(-bound, bound, size=(T, K), dtype=np.int64)
            W = rng.integers(-wb, wb, size=(N, K), dtype=np.int64)
            got = drop.matmul_exact(A, W.astype(np.float64), bound, wmax=wb)
            want = np.array([[sum(int(a) * int(b) for a, b in zip(A[i], W[j])) for j in range(N)] for i in range(T)],
                            dtype=object).astype(np.int64)
            assert np.array_equal(got, want)
    finally:
        M.close()
