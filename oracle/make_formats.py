"""Derive oracle/formats.json from the reference's format proposal (TEST INFRASTRUCTURE).

Runs only where the reference checkout is present ($EII_REFERENCE, or a directory named
`reference` beside this repository).  It restates Model.fmt (python/intref.py:154-160):
a site-layer whose class starts with "flagged" is INT32 with f = 31 - k in wide mode,
every other site is INT16 with f = 15 - k; the final norm output uses f = 15 - k(final_out|30)
(python/intref.py:296).  The 12 sites are written in model.bin's fmt[24] order
(python/export_vectors.py:34).  Narrow mode (wide=False) and the residual grid exponents of
Model._grid (python/intref.py:303-308) are kept too, and the class and k of every site-layer of the
proposal (the `prop` table a Model subclass reads in its own fmt / _grid overrides).
"""
import json, os, sys

SITES = ("norm1_out", "q_proj", "k_proj", "v_proj", "q_rope", "k_rope", "attn_ctx",
         "norm2_out", "gate_proj", "up_proj", "silu_gate", "mlp_gated")


def main():
    here = os.path.dirname(os.path.abspath(__file__))
    ref = os.environ.get("EII_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(here)), "reference")
    prop = json.load(open(os.path.join(ref, "results", "scaling_proposal.json")))["sites"]
    out = {"source": "results/scaling_proposal.json of the reference", "wide": [], "narrow": []}
    for l in range(30):
        for mode in ("wide", "narrow"):
            fm = []
            for s in SITES:
                e = prop[f"{s}|{l}"]
                flagged = e["class"].startswith("flagged")
                fm += [32, 31 - e["k"]] if (flagged and mode == "wide") else [16, 15 - e["k"]]
            out[mode].append(fm)
    out["f_y"] = 15 - prop["final_out|30"]["k"]
    out["resid_k"] = {s: [prop[f"{s}|{l}"]["k"] for l in range(30)] for s in ("resid_in", "resid_out")}
    # the class and k of every site-layer: the drop-in Model's `prop` (python/intref.py:138-139)
    out["sites"] = {name: {"class": e["class"], "k": int(e["k"])} for name, e in sorted(prop.items())}
    here = os.path.dirname(os.path.abspath(__file__))
    # one copy for the oracle, one for the engine package's synthetic-model writer
    for path in (os.path.join(here, "formats.json"),
                 os.path.join(os.path.dirname(here), "exact-integer-inference_b200", "formats.json")):
        with open(path, "w") as f:
            json.dump(out, f, indent=0)
        print("wrote", path)


if __name__ == "__main__":
    sys.exit(main())
