"""Pin the CPU oracle (oracle/) against fixtures produced by the reference itself.

tests/golden/*.json were written by tests/golden/make_golden.py, which runs the reference's own
python/intref.py and python/export_vectors.py (and its scalar C program) on the seeded synthetic
model.  Every test here is CPU-only."""
import os
import subprocess

import numpy as np
import pytest

from conftest import REPO, golden, sha256_arr, sha256_file
from oracle import forward as ofw
from oracle import synth

SETS = (("t24", "base"), ("t128", "base"), ("t160", "outlier"))


def sweep_activations(case):
    """The seeded activations make_golden.py fed the reference for a sweep case."""
    import sys
    from conftest import GOLDEN
    if GOLDEN not in sys.path:
        sys.path.insert(0, GOLDEN)
    from make_golden import gemm_activations
    return gemm_activations(case["bits_in"], case["M"], case["K"], case["act_seed"])


def test_model_bin_base_matches_reference_export(base_model_path):
    assert sha256_file(base_model_path) == golden("vectors_t24.json")["files"]["model.bin"]["sha256"]
    assert os.path.getsize(base_model_path) == 154045048


def test_model_bin_outlier_matches_reference_export(outlier_model_path):
    assert sha256_file(outlier_model_path) == golden("vectors_t160.json")["files"]["model.bin"]["sha256"]


def _states(mdl, name):
    g = golden(f"vectors_{name}.json")
    ids = synth.window_ids(g["window"], g["tokens"])
    out = ofw.forward(mdl, ids)
    return g, ids, out


@pytest.mark.parametrize("name,kind", SETS)
def test_oracle_states_match_reference(name, kind, base_model, outlier_model):
    mdl = outlier_model if kind == "outlier" else base_model
    g, ids, out = _states(mdl, name)
    files = g["files"]
    assert sha256_arr(ids, np.int64) == files["ids.i64"]["sha256"]
    assert sha256_arr(out["embed"][0], np.int32) == files["exp_embed.i32"]["sha256"]
    assert sha256_arr(out["resid"][:, 0], np.int32) == files["exp_resid_out.i32"]["sha256"]
    assert sha256_arr(out["logits"][0], np.int32) == files["exp_logits.i32"]["sha256"]
    assert out["logits"][0, 0, :8].tolist() == g["samples"]["logits_row0_first8"]


def test_negative_one_unit_change_is_detected(base_model):
    """The reference's negative test (tools/record_conformance.sh:49-69): one unit in one
    residual element must make the comparison fail."""
    g, ids, out = _states(base_model, "t24")
    res = out["resid"][:, 0].astype(np.int32).copy()
    flat = res.reshape(-1)
    flat[flat.size // 2] += 1
    assert sha256_arr(res, np.int32) != g["files"]["exp_resid_out.i32"]["sha256"]


def test_oracle_gemm_sweep_matches_reference(base_model):
    for c in golden("gemm_sweep.json")["cases"]:
        wname, wl = c["weight"]
        W = (base_model["emb_q"], base_model["emb_m"], base_model["emb_n"]) if wname == "embed" \
            else base_model["layers"][wl][wname]
        a = sweep_activations(c)
        acc = ofw.matmul_exact(a, W[0], 1 << (c["bits_in"] - 1))
        out = ofw.sat(ofw.rs(acc * W[1][None, :], W[2] + c["f_in"] - c["f_out"]), c["bits_out"])
        assert sha256_arr(acc, np.int64) == c["acc_sha256"], c["name"]
        assert sha256_arr(out, np.int64) == c["out_sha256"], c["name"]


def test_oracle_large_sweep_digests_match_reference(base_model_path):
    """The oracle's linear over the contraction sweep's seeded activations reproduces the reference's
    block digests (tests/golden/gemm_sweep_large.json) at M = 512 for all four shapes and M = 4096
    for the three layer shapes: this pins the activation generator, the digest definition and the
    formats of exact-integer-inference_b200/sweep.py that the GPU tests and bench.py use."""
    import sweep
    for c in golden("gemm_sweep_large.json")["cases"]:
        if c["M"] > (512 if c["N"] > 4096 else 4096):
            continue
        ci, M = c["case"], c["M"]
        W, m, n = sweep.weights(base_model_path, ci)
        bits_in, f_in, f_out, bits_out = sweep.case_formats(ci)
        N, K = W.shape
        a = np.concatenate([sweep.activation_block(ci, M, b, K, bits_in) for b in range(sweep.blocks(M))])
        acc = ofw.matmul_exact(a.astype(np.int64), W, 1 << (bits_in - 1))
        out = ofw.sat(ofw.rs(acc * m[None, :], n + f_in - f_out), bits_out)
        assert out[2, :8].tolist() == c["out_row2_first8"], c["name"]
        assert sweep.hexes(sweep.block_digests(sweep.row_digests(acc, N, False), M)) == c["acc_blocks"], c["name"]
        assert sweep.hexes(sweep.block_digests(sweep.row_digests(out, N, True), M)) == c["out_blocks"], c["name"]


def test_oracle_batched_subset_matches_reference(base_model):
    """Sequences of the 4096 x 128 batch, run as one batch through the oracle, reproduce the
    per-sequence logits the reference computed one sequence at a time."""
    g = golden("config4_subset.json")
    table = synth.token_table()
    seqs = g["sequences"][:4]
    ids = np.stack([table[s["row"], :g["T"]] for s in seqs])
    out = ofw.forward(base_model, ids, want_states=False)
    for s, lg in zip(seqs, out["logits"]):
        assert sha256_arr(lg, np.int32) == s["logits_i32_sha256"]


REF_BIN = os.path.join(REPO, "oracle", "_ref", "intref")


@pytest.mark.skipif(not os.path.exists(REF_BIN), reason="reference C program not built (oracle/build_ref.sh)")
def test_reference_c_program_accepts_oracle_vectors(base_model, base_model_path, tmp_path):
    """The reference's scalar C program (c/intref.c) checks vectors written by the oracle."""
    g, ids, out = _states(base_model, "t24")
    ids.astype(np.int64).tofile(tmp_path / "ids.i64")
    out["embed"][0].astype(np.int32).tofile(tmp_path / "exp_embed.i32")
    out["resid"][:, 0].astype(np.int32).tofile(tmp_path / "exp_resid_out.i32")
    out["logits"][0].astype(np.int32).tofile(tmp_path / "exp_logits.i32")
    os.symlink(base_model_path, tmp_path / "model.bin")
    r = subprocess.run([REF_BIN, str(tmp_path)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL STATES EXACT" in r.stdout


def test_silu_tables_obey_the_odd_part_identity(base_model):
    """silu(x) - silu(-x) = x, so each rounded table satisfies tab[g] = SAT(tab[-g] + g 2^(f_s-f_g))
    for g > 0 when f_s >= f_g; the engine keeps only the negative half in shared memory when this
    holds for every input (and verifies it itself at load)."""
    checked = 0
    for Ly in base_model["layers"]:
        F = ofw.fm_unpack(Ly["fm"])
        (_, f_g), (bits_s, f_s) = F["g"], F["s"]
        d = f_s - f_g
        if d < 0:
            continue
        tab = np.asarray(Ly["silu"], dtype=np.int64)
        g = np.arange(1, 32768, dtype=np.int64)
        pred = ofw.sat(tab[32768 - g] + (g << d), bits_s)
        assert np.array_equal(pred, tab[32768 + g])
        checked += 1
    assert checked == 30


def trace_inputs(mdl):
    """The t24 residual entering each layer of the trace fixture (oracle forward, itself pinned)."""
    g = golden("trace_t24.json")
    ids = synth.window_ids(g["window"], g["tokens"])
    x = ofw.embed(mdl, ids)
    out = {}
    for l in range(max(int(k) for k in g["layers"]) + 1):
        if str(l) in g["layers"]:
            out[l] = x.copy()
        x = ofw.block_batch(mdl, l, x, g["tokens"])
    return g, out


def check_trace(tr, want):
    """Every site of a block trace against the reference's digests (and the exponents)."""
    assert {k: int(v) for k, v in tr["_f"].items()} == want["f"]
    bad = []
    for k, s in want["sites"].items():
        a = np.ascontiguousarray(tr[k], dtype=np.int64)
        if list(a.shape) != s["shape"] or sha256_arr(a, np.int64) != s["sha256"]:
            bad.append(k)
    assert not bad, bad
    assert set(tr) - {"_f"} == set(want["sites"])


def test_oracle_block_trace_matches_reference(base_model):
    """Per-site trace of Model.block (python/intref.py:192-286) on the t24 tokens at five layers."""
    g, xs = trace_inputs(base_model)
    for l, x in xs.items():
        tr = {}
        ofw.block_batch(base_model, l, x, g["tokens"], trace=tr)
        check_trace(tr, g["layers"][str(l)])
