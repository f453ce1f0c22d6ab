"""Time the reference's own scalar C program (c/intref.c, built into oracle/_ref/intref by
oracle/build_ref.sh) on BASELINE configs 1-3, one process per config, on this host.

TEST/MEASUREMENT INFRASTRUCTURE.  The vector directories are written from the oracle (oracle/forward.py,
pinned to the reference's export digests) in python/export_vectors.py's layout; the program checks
every state against them (ALL STATES EXACT) and reports its own time, which excludes the model load
(c/intref.c:225,256).

    python oracle/time_reference_c.py [--out FILE]
"""
import argparse
import json
import os
import re
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "tests"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    import bench
    from conftest import ensure_model, golden
    from oracle import forward as ofw
    from oracle import synth
    from oracle.modelbin import read_model_bin
    ref = os.path.join(HERE, "_ref", "intref")
    if not os.path.exists(ref):
        raise SystemExit("oracle/_ref/intref not built (sh oracle/build_ref.sh REFERENCE_DIR)")
    res = {"program": "reference c/intref.c -O2, one process, its own timer", "runs": {}}
    with tempfile.TemporaryDirectory() as td:
        for key, name, kind in (("config1_t24", "t24", "base"), ("config2_t128", "t128", "base"),
                                ("config3_t160_outlier", "t160", "outlier")):
            g = golden(f"vectors_{name}.json")
            path = ensure_model(kind)
            ids = synth.window_ids(g["window"], g["tokens"])
            out = ofw.forward(read_model_bin(path), ids)
            d = bench.write_vector_dirs(os.path.join(td, name), path,
                                        [(ids, out["embed"][0], out["resid"][:, 0], out["logits"][0])])[0]
            o = subprocess.run([ref, d], capture_output=True, text=True).stdout.strip().splitlines()[-1]
            m = re.search(r"\((\d+) tokens, ([0-9.]+) s\)", o)
            secs = float(m.group(2)) if m else None
            res["runs"][key] = {"T": int(g["tokens"]), "seconds": secs,
                                "tokens_per_s": round(g["tokens"] / secs, 2) if secs else None, "verdict": o}
    text = json.dumps(res, indent=1)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text + "\n")
    print(text)


if __name__ == "__main__":
    main()
