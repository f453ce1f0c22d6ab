"""Seeded synthetic SmolLM2-135M model and token windows (TEST INFRASTRUCTURE: oracle only).

The real checkpoint and wikitext are not available, so parity runs on a synthetic model of the
same architecture.  Float weights are N(0, 0.02^2) float32 drawn from ONE
np.random.default_rng(seed) in the fixed order embed [49152,576], then per layer q, k, v, o,
gate, up, down; RMSNorm gains are 1.0, and the "outlier" variant scales channels
OUTLIER_CHANNELS of every ln1/ln2/final gain by 50.  They are quantised exactly as the
reference quantiser does:

  quant_rows       python/intref.py:113-123   per-row int8 + (m, n), m in [2^13, 2^14]
  quant_vec_int16  python/intref.py:126-130   gain vector -> (int16 q, f)

and written, with the formats of oracle/formats.json (Model.fmt, intref.py:154-160) and the
exact tables of oracle/tables.py, to model.bin in the layout of c/intref.c:8-13 (writer
python/export_vectors.py:24-45).  Token windows: rng(ids_seed).integers(0, 49152, (rows, 512));
sequence `window` is row `window`, first T ids (python/export_vectors.py:16-17 takes
wins[win][:T] of the tokenised wikitext windows in the same way).
"""
import json
import math
import os

import numpy as np

from . import tables
from .modelbin import D, DFF, LIN_NAMES, LIN_SHAPES, NL, V, write_model_bin

WEIGHT_SEED = 0
IDS_SEED = 1
IDS_ROWS = 4096
OUTLIER_CHANNELS = (7, 101, 333, 507)
OUTLIER_GAIN = 50.0
HERE = os.path.dirname(os.path.abspath(__file__))


def load_formats(mode="wide"):
    with open(os.path.join(HERE, "formats.json")) as f:
        j = json.load(f)
    return [list(x) for x in j[mode]], int(j["f_y"]), j


def float_weights(seed=WEIGHT_SEED, outlier=False):
    """Float32 weights in the dict shape of python/common.py:50-68 (numpy instead of torch)."""
    rng = np.random.default_rng(seed)
    sd = np.float32(0.02)

    def draw(shape):
        return rng.standard_normal(shape, dtype=np.float32) * sd

    W = {"embed": draw((V, D)), "layers": []}
    for _ in range(NL):
        Ly = {}
        for nm in LIN_NAMES:
            Ly[nm] = draw(LIN_SHAPES[nm])
        W["layers"].append(Ly)
    gain = np.ones(D, dtype=np.float32)
    if outlier:
        gain[list(OUTLIER_CHANNELS)] = np.float32(OUTLIER_GAIN)
    W["norm"] = gain.copy()
    for Ly in W["layers"]:
        Ly["ln1"] = gain.copy()
        Ly["ln2"] = gain.copy()
    return W


def quant_rows(W):
    # python/intref.py:113-123
    W = W.astype(np.float64)
    s = np.abs(W).max(1) / 127.0
    s = np.where(s == 0, 1.0, s)
    n = (13 - np.floor(np.log2(s))).astype(np.int64)
    m = np.rint(s * 2.0 ** n).astype(np.int64)
    if not (m.min() >= 2 ** 13 and m.max() <= 2 ** 14):
        raise ValueError("row multiplier out of [2^13, 2^14]")
    sw = m * 2.0 ** (-n.astype(np.float64))
    q = np.clip(np.rint(W / sw[:, None]), -127, 127)
    return q.astype(np.int8), m, n


def quant_vec_int16(w):
    # python/intref.py:126-130
    w = w.astype(np.float64)
    f = 14 - int(math.floor(math.log2(np.abs(w).max())))
    q = np.clip(np.rint(w * 2.0 ** f), -32768, 32767).astype(np.int64)
    return q, f


def build_model(seed=WEIGHT_SEED, outlier=False, mode="wide", procs=None, silu_cache=None):
    """Quantised model dict (write_model_bin shape).  silu_cache maps (f_in, f_out, bits) ->
    table and is filled in place so several variants share the mpmath work."""
    fms, f_y, _ = load_formats(mode)
    W = float_weights(seed, outlier)
    mdl = {}
    mdl["emb_q"], mdl["emb_m"], mdl["emb_n"] = quant_rows(W["embed"])
    mdl["final_q"], mdl["final_f"] = quant_vec_int16(W["norm"])
    mdl["f_y"] = f_y
    mdl["exp"] = tables.exp_table()
    mdl["rope_c"], mdl["rope_s"] = tables.rope_tables(512)
    keys = []
    for l in range(NL):
        fm = fms[l]
        f_g, bits_s, f_s = fm[17], fm[20], fm[21]
        keys.append((f_g, f_s, bits_s))
    cache = silu_cache if silu_cache is not None else {}
    missing = [k for k in set(keys) if k not in cache]
    cache.update(tables.silu_tables_parallel(missing, procs))
    layers = []
    for l, Lw in enumerate(W["layers"]):
        Ly = {"fm": np.asarray(fms[l], dtype=np.int64)}
        Ly["ln1_q"], Ly["ln1_f"] = quant_vec_int16(Lw["ln1"])
        Ly["ln2_q"], Ly["ln2_f"] = quant_vec_int16(Lw["ln2"])
        for nm in LIN_NAMES:
            Ly[nm] = quant_rows(Lw[nm])
        Ly["silu"] = cache[keys[l]]
        layers.append(Ly)
    mdl["layers"] = layers
    return mdl


def token_table(rows=IDS_ROWS, seed=IDS_SEED):
    return np.random.default_rng(seed).integers(0, V, size=(rows, 512), dtype=np.int64)


def window_ids(window, T, rows=IDS_ROWS, seed=IDS_SEED):
    return token_table(max(rows, window + 1), seed)[window, :T].copy()


def write_synthetic(path, seed=WEIGHT_SEED, outlier=False, procs=None, silu_cache=None):
    mdl = build_model(seed, outlier, procs=procs, silu_cache=silu_cache)
    write_model_bin(path, mdl)
    return mdl
