"""Time the reference's own numpy engine (python/intref.py `Model.forward`, :288-301) on this host's
CPU, for BASELINE configs 1-3 and the 64-sequence check subset of config 4.

TEST/MEASUREMENT INFRASTRUCTURE, not part of the engine.  The reference's Python module is imported
from its checkout (`--reference DIR` or $EII_REFERENCE; it is never copied into this repository and
does not travel to the GPU host), with its two loaders patched to the seeded synthetic weights and
token table exactly as tests/golden/make_golden.py does.  Table and model construction (mpmath) are
excluded from the timing (an untimed 8-token forward first builds the tables the reference makes
lazily), as the reference's C program excludes its model load (c/intref.c:225).

    python oracle/time_reference_numpy.py --reference DIR [--threads N ...] [--subset K] [--repeat R] [--out FILE]

One process per BLAS thread count (OPENBLAS_NUM_THREADS etc. are set before numpy loads).  Configs
1-3 are timed R times (best kept); the subset once.  Every timed forward's logits are compared with
the golden digests the reference produced (tests/golden), so the timed runs are checked runs.
"""
import argparse
import hashlib
import json
import os
import platform
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def child(ref, subset_n, repeat):
    sys.path.insert(0, REPO)
    sys.path.insert(0, os.path.join(REPO, "tests", "golden"))
    import numpy as np
    import make_golden as mg
    os.environ["EII_REFERENCE"] = ref
    torch, common, intref = mg.import_reference()
    from oracle import synth

    def golden(name):
        with open(os.path.join(REPO, "tests", "golden", name)) as f:
            return json.load(f)

    def sha(logits):
        return hashlib.sha256(np.ascontiguousarray(logits, dtype=np.int32).tobytes()).hexdigest()

    out = {}
    for outlier, sets in ((False, (("config1_t24", "t24"), ("config2_t128", "t128"))),
                          (True, (("config3_t160_outlier", "t160"),))):
        mg.patch(torch, common, intref, outlier)
        M = intref.Model(wide=True)
        M.forward(synth.window_ids(0, 8))  # untimed
        for key, name in sets:
            g = golden(f"vectors_{name}.json")
            ids = synth.window_ids(g["window"], g["tokens"])
            best, ok = None, True
            for _ in range(repeat):
                t0 = time.perf_counter()
                logits = M.forward(ids)
                dt = time.perf_counter() - t0
                best = dt if best is None else min(best, dt)
                ok = ok and sha(logits) == g["files"]["exp_logits.i32"]["sha256"]
            out[key] = {"T": int(g["tokens"]), "seconds": round(best, 3), "tokens_per_s": round(g["tokens"] / best, 2),
                        "repeats": repeat, "logits_equal_golden": ok}
        if not outlier and subset_n:
            g = golden("config4_subset.json")
            seqs = g["sequences"][:subset_n]
            table = synth.token_table()
            ok = 0
            t0 = time.perf_counter()
            for s in seqs:
                ok += sha(M.forward(table[s["row"], :g["T"]])) == s["logits_i32_sha256"]
            dt = time.perf_counter() - t0
            out["config4_subset"] = {"sequences": len(seqs), "T": g["T"], "seconds": round(dt, 2),
                                     "tokens_per_s": round(len(seqs) * g["T"] / dt, 2), "logits_equal_golden": ok}
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EII_REFERENCE"))
    ap.add_argument("--threads", type=int, nargs="*", default=None, help="BLAS thread counts (default: 1 and all)")
    ap.add_argument("--subset", type=int, default=64, help="config-4 check-subset sequences to time")
    ap.add_argument("--repeat", type=int, default=3, help="timed forwards per config 1-3 (best kept)")
    ap.add_argument("--out", default=None)
    ap.add_argument("--child", action="store_true", help=argparse.SUPPRESS)
    a = ap.parse_args()
    if not a.reference or not os.path.isdir(os.path.join(a.reference, "python")):
        raise SystemExit("the reference checkout is needed: --reference DIR or EII_REFERENCE")
    if a.child:
        child(a.reference, a.subset, a.repeat)
        return
    threads = a.threads or [1, os.cpu_count()]
    res = {"cpu": cpu_model(), "nproc": os.cpu_count(), "numpy_path": "reference python/intref.py Model.forward",
           "runs": {}}
    for n in threads:
        env = dict(os.environ)
        for k in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS"):
            env[k] = str(n)
        p = subprocess.run([sys.executable, os.path.abspath(__file__), "--child", "--reference", a.reference,
                            "--subset", str(a.subset), "--repeat", str(a.repeat)],
                           env=env, capture_output=True, text=True, check=True)
        res["runs"][f"{n}_threads"] = json.loads(p.stdout.strip().splitlines()[-1])
    text = json.dumps(res, indent=1)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text + "\n")
    print(text)


if __name__ == "__main__":
    main()
