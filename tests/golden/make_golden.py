"""Generate the golden fixtures in tests/golden/ by running the REFERENCE itself.

Runs only where the reference checkout is present: $EII_REFERENCE, or a directory named
`reference` beside this repository.  The fixtures it writes are committed so the tests never need
the reference.

What it does, for the seeded synthetic model of oracle/synth.py:
  1. imports the reference's python/intref.py and python/common.py, and patches the two loader
     names intref.load_config / intref.load_weights (imported at python/intref.py:31) and
     common.load_token_windows (python/common.py:71) so they return the seeded synthetic
     weights and token table instead of the HF checkpoint and wikitext;
  2. runs the reference's own python/export_vectors.py (runpy) for the three vector sets of the
     reference (t24: window 64, 24 tokens; t128: window 64, 128 tokens; t160: window 100,
     160 tokens, here on the outlier-gain model) and records the size and sha256 of model.bin and
     of every exported state, like vectors/*/manifest.json;
  3. runs the reference's scalar C program (oracle/_ref/intref, built by oracle/build_ref.sh)
     on each set and records its verdict line;
  4. runs intref.Model.forward on the 64-sequence check subset of the 4096-sequence batch
     (T=128) and records per-sequence sha256 digests of the int32 logits and last residual;
  5. runs intref.Model.linear / matmul_exact + rs on seeded activations spanning the full
     INT16 / INT32 ranges for the four contraction shapes and records digests of acc and out;
  6. runs intref.Model.block(l, x, trace) on the t24 tokens for the layers in TRACE_LAYERS and
     records the sha256 of every trace site (int64, C order) and the site exponents (trace_t24.json);
  7. runs intref.Model(wide).forward(ids, narrow_residual) on the t24 tokens for the narrow comparison
     modes and records the logits digests (narrow_t24.json);
  8. records digests of the reference's exp, RoPE and SiLU tables for every format pair of its
     format table (tables.json);
  8b. runs Model subclasses of the reference with the overrides its ablation scripts use
     (python/ablate_narrow.py:30-40 fmt, ablate_perchannel.py:21-36 and ablate_layers.py:27-44
     _grid) on the t24 tokens and records the logits digests (ablation_t24.json);
  9. runs intref.Model.linear on the contraction sweep of exact-integer-inference_b200/sweep.py
     (four weight shapes, M = 512 ... 262144 rows, seeded activations over the full INT16 / INT32
     ranges) and records the block digests of acc and of the requantised outputs
     (gemm_sweep_large.json; about ten minutes of numpy).

    python tests/golden/make_golden.py [--keep DIR] [--skip-subset] [--only-trace] [--only-narrow]
                                       [--only-tables] [--only-sweep] [--only-ablation]
"""
import argparse
import hashlib
import json
import os
import runpy
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)
from oracle import synth  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_dir():
    """The reference checkout: $EII_REFERENCE, else `reference` beside this repository."""
    ref = os.environ.get("EII_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference")
    if not os.path.isdir(os.path.join(ref, "python")):
        raise SystemExit(f"reference checkout not found at {ref} (set EII_REFERENCE)")
    return ref


REF = None
SETS = (("t24", 64, 24, False), ("t128", 64, 128, False), ("t160", 100, 160, True))
SUBSET_SEED = 2
SUBSET_N = 64
TRACE_LAYERS = (0, 4, 11, 13, 28)


def sha256_bytes(b):
    return hashlib.sha256(b).hexdigest()


def sha256_file(p):
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def import_reference():
    global REF
    import torch
    REF = reference_dir()
    sys.path.insert(0, os.path.join(REF, "python"))
    import common
    import intref
    return torch, common, intref


def patch(torch, common, intref, outlier):
    W = synth.float_weights(synth.WEIGHT_SEED, outlier)
    tW = {"embed": torch.from_numpy(W["embed"]), "norm": torch.from_numpy(W["norm"]), "layers": []}
    for Ly in W["layers"]:
        tW["layers"].append({k: torch.from_numpy(v) for k, v in Ly.items()})
    intref.load_config = lambda: {"num_hidden_layers": 30}
    intref.load_weights = lambda: tW
    table = synth.token_table()
    common.load_token_windows = lambda: (table, {})


def subset_rows():
    return sorted(np.random.default_rng(SUBSET_SEED).choice(synth.IDS_ROWS, SUBSET_N, replace=False).tolist())


def gemm_cases():
    """(name, weight source, site-layer for (f_in, bits_in), out format, M) for the sweep."""
    return [
        ("q_576x576", ("q", 0), "norm1_out|0", ("q_proj", 0), 512),
        ("gate_1536x576", ("gate", 11), "norm2_out|11", ("gate_proj", 11), 1000),
        ("down_576x1536", ("down", 0), "mlp_gated|0", ("resid", 15), 700),
        ("down16_576x1536", ("down", 3), "mlp_gated|3", ("resid", 15), 512),
        ("logits_49152x576", ("embed", None), "final_out|30", ("logits", 16), 160),
    ]


def gemm_activations(bits, M, K, seed):
    rng = np.random.default_rng(seed)
    lo, hi = -(1 << (bits - 1)), (1 << (bits - 1))
    a = rng.integers(lo, hi, size=(M, K), dtype=np.int64)
    a[0, :] = lo          # extreme rows exercise the full range exactly
    a[1, :] = hi - 1
    return a


def trace_golden(torch, common, intref):
    """Digests of the reference's per-site block trace (python/intref.py:192-286) on the t24 tokens."""
    patch(torch, common, intref, False)
    M_ = intref.Model(wide=True)
    ids = synth.window_ids(64, 24)
    x = M_.embed(ids)
    layers = {}
    for l in range(max(TRACE_LAYERS) + 1):
        if l in TRACE_LAYERS:
            tr = {}
            x_next = M_.block(l, x, trace=tr)
            layers[str(l)] = {"f": {k: int(v) for k, v in tr["_f"].items()},
                              "sites": {k: {"shape": list(np.shape(v)),
                                            "sha256": sha256_bytes(np.ascontiguousarray(v, dtype=np.int64).tobytes())}
                                        for k, v in tr.items() if k != "_f"}}
            x = x_next
        else:
            x = M_.block(l, x)
        print("trace layer", l, "done", flush=True)
    with open(os.path.join(HERE, "trace_t24.json"), "w") as f:
        json.dump({"window": 64, "tokens": 24, "model": "base", "note": "sha256 of int64 C-order arrays of "
                   "Model.block(l, x, trace) sites; x is the reference's own residual entering layer l",
                   "layers": layers}, f, indent=1)


def narrow_golden(torch, common, intref):
    """Logits digests of the reference's narrow comparison modes (python/intref.py:152-160,288-308) on
    the t24 tokens: formats narrowed (wide=False) with and without the residual grid, and the residual
    grid alone (wide=True)."""
    patch(torch, common, intref, False)
    ids = synth.window_ids(64, 24)
    out = {}
    for wide, nres in ((False, False), (False, True), (True, True)):
        M_ = intref.Model(wide=wide)
        lg = M_.forward(ids, narrow_residual=nres)
        out[f"wide={int(wide)},narrow_residual={int(nres)}"] = {
            "logits_int64_sha256": sha256_bytes(np.ascontiguousarray(lg, dtype=np.int64).tobytes()),
            "logits_row0_first8": np.asarray(lg[0, :8]).tolist()}
        print("narrow", wide, nres, "done", flush=True)
    with open(os.path.join(HERE, "narrow_t24.json"), "w") as f:
        json.dump({"window": 64, "tokens": 24, "model": "base", "note": "Model(wide).forward(ids, narrow_residual) "
                   "int64 logits [T, 49152] of the reference", "modes": out}, f, indent=1)


ABLATION_SEED = 31


def ablation_shifts():
    """Per-channel residual-grid shifts of the per-channel variant: {(site, l): int64 [576]} in [2, 8]
    from a seeded generator (the reference derives them from calibration maxima, which are not
    available here; the grid arithmetic is the same)."""
    rng = np.random.default_rng(ABLATION_SEED)
    return {(site, l): rng.integers(2, 9, size=576).astype(np.int64) for site in ("resid_in", "resid_out")
            for l in range(30)}


def ablation_golden(torch, common, intref):
    """Logits digests of reference Model subclasses with the overrides of its ablation scripts, t24."""
    patch(torch, common, intref, False)
    ids = synth.window_ids(64, 24)
    F_RES = intref.F_RES

    class NarrowSites(intref.Model):
        """fmt: flagged sites stay INT32 unless narrow mode names them (ablate_narrow.py:30-40)."""
        narrow_sites = None

        def fmt(self, site, l):
            e = self.prop[f"{site}|{l}"]
            if e["class"].startswith("flagged"):
                if self.wide or (self.narrow_sites is not None and site not in self.narrow_sites):
                    return 32, 31 - e["k"]
            return 16, 15 - e["k"]

    pcs = ablation_shifts()

    class ChannelGrid(intref.Model):
        """_grid with one shift per channel (ablate_perchannel.py:31-36)."""
        def _grid(self, x, site, l):
            s = pcs[(site, l)][None, :]
            half = np.where(s > 0, np.int64(1) << np.maximum(s - 1, 0), 0)
            y = np.where(s > 0, (x + half) >> s, x)
            return intref.sat(y, 16) << s

    class SomeLayers(intref.Model):
        """_grid applied at layers 12..28 only (ablate_layers.py:31-34)."""
        def _grid(self, x, site, l):
            return super()._grid(x, site, l) if 12 <= l < 29 else x

    out = {}
    M_ = NarrowSites(wide=False)
    for name, sites in (("flagged_gated_only", {"mlp_gated"}), ("flagged_ctx_silu_only", {"attn_ctx", "silu_gate"})):
        M_.narrow_sites = sites
        lg = M_.forward(ids)
        out[name] = {"logits_int64_sha256": sha256_bytes(np.ascontiguousarray(lg, dtype=np.int64).tobytes()),
                     "logits_row0_first8": np.asarray(lg[0, :8]).tolist()}
        print("ablation", name, flush=True)
    for name, cls in (("channel_grid", ChannelGrid), ("grid_layers_12_28", SomeLayers)):
        lg = cls(wide=True).forward(ids, narrow_residual=True)
        out[name] = {"logits_int64_sha256": sha256_bytes(np.ascontiguousarray(lg, dtype=np.int64).tobytes()),
                     "logits_row0_first8": np.asarray(lg[0, :8]).tolist()}
        print("ablation", name, flush=True)
    with open(os.path.join(HERE, "ablation_t24.json"), "w") as f:
        json.dump({"window": 64, "tokens": 24, "model": "base", "channel_grid_seed": ABLATION_SEED,
                   "note": "int64 logits [T, 49152] of reference Model subclasses (fmt / _grid overrides of its "
                           "ablation scripts); channel_grid shifts: rng(seed).integers(2, 9, 576) per (site, layer), "
                           "resid_in layers 0..29 then resid_out layers 0..29", "variants": out}, f, indent=1)


def tables_golden(intref):
    """Digests of the reference's own mpmath tables (python/intref.py:66-108): exp_table(),
    rope_tables(512) and silu_table(f_g, f_s, bits_s) for every (gate, silu) format pair of the
    reference's format table, wide and narrow modes (oracle/formats.json)."""
    with open(os.path.join(REPO, "oracle", "formats.json")) as f:
        fmt = json.load(f)
    keys = sorted({(fm[17], fm[21], fm[20]) for mode in ("wide", "narrow") for fm in fmt[mode]})
    out = {"exp": sha256_bytes(np.ascontiguousarray(intref.exp_table(), dtype=np.int64).tobytes())}
    C, S = intref.rope_tables(512)
    out["rope_cos"] = sha256_bytes(np.ascontiguousarray(C, dtype=np.int64).tobytes())
    out["rope_sin"] = sha256_bytes(np.ascontiguousarray(S, dtype=np.int64).tobytes())
    out["silu"] = {f"{fi},{fo},{b}": sha256_bytes(np.ascontiguousarray(intref.silu_table(fi, fo, b), dtype=np.int64).tobytes())
                   for fi, fo, b in keys}
    with open(os.path.join(HERE, "tables.json"), "w") as f:
        json.dump({"note": "sha256 of int64 C-order tables from the reference's own python/intref.py functions "
                   "(mpmath 50 digits); silu keys are f_in,f_out,bits", "tables": out}, f, indent=1)
    print("tables done:", len(keys), "SiLU keys", flush=True)


_SWEEP_JOB = {}


def _sweep_block(b):
    """Row digests of block b of the current sweep case through the reference's Model.linear."""
    j = _SWEEP_JOB
    sweep = j["sweep"]
    a_blk = sweep.activation_block(j["ci"], j["M"], b, j["K"], j["bits_in"]).astype(np.int64)
    step = 1024 if j["N"] > 4096 else sweep.BLOCK
    da, do, first8 = [], [], None
    for r in range(0, a_blk.shape[0], step):
        out, acc = j["linear"](a_blk[r:r + step], 1 << (j["bits_in"] - 1), j["W"], j["f_in"], j["f_out"], j["bits_out"])
        da.append(sweep.row_digests(acc, j["N"], False))
        do.append(sweep.row_digests(out, j["N"], True))
        if first8 is None:
            first8 = np.asarray(out[2, :8]).tolist()
    return np.concatenate(da), np.concatenate(do), first8


def sweep_golden(torch, common, intref):
    """Block digests of the reference's Model.linear (python/intref.py:186-190) over the contraction
    sweep of sweep.py: acc (the exact int64 matmul_exact) and out = SAT(RS(acc m, n + f_in - f_out))."""
    sys.path.insert(0, os.path.join(REPO, "exact-integer-inference_b200"))
    import sweep
    patch(torch, common, intref, False)
    M_ = intref.Model(wide=True)
    cases = []
    for ci, (name, (wname, wl), (si, li), outs) in enumerate(sweep.CASES):
        W = (M_.emb_q, M_.emb_m, M_.emb_n) if wname == "embed" else M_.layers[wl][wname]
        if si == "final_out":
            bits_in, f_in = 16, 15 - M_.prop["final_out|30"]["k"]
        else:
            bits_in, f_in = M_.fmt(si, li)
        if outs[0] == "grid":
            f_out, bits_out = outs[1], outs[2]
        else:
            bits_out, f_out = M_.fmt(outs[0], outs[1])
        assert (bits_in, f_in, f_out, bits_out) == sweep.case_formats(ci), name
        N, K = W[0].shape
        for M in sweep.MS:
            t0 = time.time()
            dacc = np.empty(M, np.uint64)
            dout = np.empty(M, np.uint64)
            _SWEEP_JOB.update(ci=ci, M=M, K=K, N=N, W=W, bits_in=bits_in, f_in=f_in, f_out=f_out, bits_out=bits_out,
                              linear=M_.linear, sweep=sweep)
            nb = sweep.blocks(M)
            if nb > 1:  # blocks in forked workers (no GPU here); numpy's elementwise passes are single-threaded
                import multiprocessing as mp
                with mp.get_context("fork").Pool(min(nb, 6)) as pool:
                    res = pool.map(_sweep_block, range(nb))
            else:
                res = [_sweep_block(0)]
            first8 = res[0][2]
            for b, (da, do, _) in enumerate(res):
                dacc[sweep.BLOCK * b:sweep.BLOCK * b + len(da)] = da
                dout[sweep.BLOCK * b:sweep.BLOCK * b + len(do)] = do
            ba, bo = sweep.block_digests(dacc, M), sweep.block_digests(dout, M)
            cases.append({"name": name, "case": ci, "M": M, "N": int(N), "K": int(K), "bits_in": bits_in, "f_in": f_in,
                          "f_out": f_out, "bits_out": bits_out, "acc": f"{sweep.total(ba):016x}",
                          "out": f"{sweep.total(bo):016x}", "acc_blocks": sweep.hexes(ba), "out_blocks": sweep.hexes(bo),
                          "out_row2_first8": first8, "seconds": round(time.time() - t0, 1)})
            print(name, M, round(time.time() - t0, 1), "s", flush=True)
    with open(os.path.join(HERE, "gemm_sweep_large.json"), "w") as f:
        json.dump({"note": "digests (hex, mod 2^64) defined in exact-integer-inference_b200/sweep.py, of the reference's "
                   "Model.linear on the sweep's seeded activations", "seed": sweep.SEED, "block_rows": sweep.BLOCK,
                   "cases": cases}, f, indent=1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--keep", default=None, help="directory to keep the exported vector sets in")
    ap.add_argument("--skip-subset", action="store_true")
    ap.add_argument("--only-trace", action="store_true")
    ap.add_argument("--only-narrow", action="store_true")
    ap.add_argument("--only-tables", action="store_true")
    ap.add_argument("--only-sweep", action="store_true")
    ap.add_argument("--only-ablation", action="store_true")
    args = ap.parse_args()
    torch, common, intref = import_reference()
    if args.only_sweep:
        sweep_golden(torch, common, intref)
        return
    if args.only_ablation:
        ablation_golden(torch, common, intref)
        return
    if args.only_tables:
        tables_golden(intref)
        return
    if args.only_trace:
        trace_golden(torch, common, intref)
        return
    if args.only_narrow:
        narrow_golden(torch, common, intref)
        return
    out_root = args.keep or tempfile.mkdtemp(prefix="eii_golden_")
    refbin = os.path.join(REPO, "oracle", "_ref", "intref")
    if not os.path.exists(refbin):
        subprocess.check_call(["sh", os.path.join(REPO, "oracle", "build_ref.sh"), REF])
    export = os.path.join(REF, "python", "export_vectors.py")

    for name, win, T, outlier in SETS:
        patch(torch, common, intref, outlier)
        d = os.path.join(out_root, name)
        t0 = time.time()
        argv = sys.argv
        sys.argv = [export, d, str(win), str(T)]
        try:
            runpy.run_path(export, run_name="__main__")
        finally:
            sys.argv = argv
        man = {"window": win, "tokens": T, "model": "outlier" if outlier else "base",
               "weight_seed": synth.WEIGHT_SEED, "ids_seed": synth.IDS_SEED, "files": {}}
        for fn in ("model.bin", "ids.i64", "exp_embed.i32", "exp_resid_out.i32", "exp_logits.i32"):
            p = os.path.join(d, fn)
            man["files"][fn] = {"bytes": os.path.getsize(p), "sha256": sha256_file(p)}
        lg = np.fromfile(os.path.join(d, "exp_logits.i32"), dtype=np.int32).reshape(T, -1)
        rz = np.fromfile(os.path.join(d, "exp_resid_out.i32"), dtype=np.int32).reshape(30, T, -1)
        man["samples"] = {"logits_row0_first8": lg[0, :8].tolist(), "logits_last_first8": lg[-1, :8].tolist(),
                          "logits_absmax": int(np.abs(lg.astype(np.int64)).max()),
                          "resid29_last_first8": rz[29, -1, :8].tolist()}
        r = subprocess.run([refbin, d], capture_output=True, text=True)
        man["reference_c"] = {"returncode": r.returncode, "last_line": r.stdout.strip().splitlines()[-1]}
        man["export_seconds"] = round(time.time() - t0, 1)
        with open(os.path.join(HERE, f"vectors_{name}.json"), "w") as f:
            json.dump(man, f, indent=1)
        print(name, man["reference_c"], man["export_seconds"], "s", flush=True)

    # GEMM sweep fixtures (base model)
    patch(torch, common, intref, False)
    M_ = intref.Model(wide=True)
    cases = []
    for i, (name, (wname, wl), site_in, (site_out, lo), Mrows) in enumerate(gemm_cases()):
        if wname == "embed":
            W = (M_.emb_q, M_.emb_m, M_.emb_n)
            bits_in, f_in = 16, 15 - M_.prop["final_out|30"]["k"]
        else:
            W = M_.layers[wl][wname]
            s, l = site_in.split("|")
            bits_in, f_in = M_.fmt(s, int(l))
        K = W[0].shape[1]
        a = gemm_activations(bits_in, Mrows, K, seed=100 + i)
        if site_out in ("resid", "logits"):
            f_out, bits_out = lo, 64
            acc = intref.matmul_exact(a, W[0], 1 << (bits_in - 1))
            out = intref.rs(acc * W[1][None, :], W[2] + f_in - f_out)
        else:
            bits_out, f_out = M_.fmt(site_out, lo)
            out, acc = M_.linear(a, 1 << (bits_in - 1), W, f_in, f_out, bits_out)
        cases.append({"name": name, "weight": [wname, wl], "bits_in": bits_in, "f_in": f_in,
                      "f_out": f_out, "bits_out": bits_out, "M": Mrows, "N": int(W[0].shape[0]), "K": int(K),
                      "act_seed": 100 + i,
                      "acc_sha256": sha256_bytes(np.ascontiguousarray(acc, dtype=np.int64).tobytes()),
                      "out_sha256": sha256_bytes(np.ascontiguousarray(out, dtype=np.int64).tobytes()),
                      "out_first8": np.asarray(out[2, :8]).tolist()})
        print(name, "done", flush=True)
    with open(os.path.join(HERE, "gemm_sweep.json"), "w") as f:
        json.dump({"note": "acc/out digests are over little-endian int64 arrays [M,N]", "cases": cases}, f, indent=1)

    if not args.skip_subset:
        rows = subset_rows()
        table = synth.token_table()
        T = 128
        seqs = []
        t0 = time.time()
        for r in rows:
            ids = table[r, :T]
            x = M_.embed(ids)
            for l in range(M_.L):
                x = M_.block(l, x)
            bits_y, f_y = 16, 15 - M_.prop["final_out|30"]["k"]
            y = M_.rmsnorm(x, M_.final_gain, f_y, bits_y)
            acc = intref.matmul_exact(y, M_.emb_q, 1 << 15)
            lg = intref.rs(acc * M_.emb_m[None, :], M_.emb_n + f_y - 16)
            seqs.append({"row": r, "logits_i32_sha256": sha256_bytes(lg.astype(np.int32).tobytes()),
                         "resid29_i32_sha256": sha256_bytes(x.astype(np.int32).tobytes()),
                         "argmax_last": int(lg[-1].argmax())})
        with open(os.path.join(HERE, "config4_subset.json"), "w") as f:
            json.dump({"T": T, "subset_seed": SUBSET_SEED, "rows": rows, "sequences": seqs,
                       "seconds": round(time.time() - t0, 1)}, f, indent=1)
        print("subset done", round(time.time() - t0, 1), "s")
    trace_golden(torch, common, intref)
    narrow_golden(torch, common, intref)
    ablation_golden(torch, common, intref)
    tables_golden(intref)
    print("vector sets in", out_root)


if __name__ == "__main__":
    main()
