"""Seeded synthetic SmolLM2-135M in the reference's model.bin format (benchmark input data).

The real checkpoint is not available here, so the benchmark and smoke runs use a synthetic model
of the same architecture, quantised exactly the way the reference's exporter does it:

  float weights  N(0, 0.02^2) float32 from one np.random.default_rng(seed), drawn in the order
                 embed [49152,576], then per layer q, k, v, o, gate, up, down; RMSNorm gains 1.0
                 (the "outlier" variant scales channels 7, 101, 333, 507 of every gain by 50)
  quantiser      per-row int8 with m in [2^13, 2^14] (python/intref.py:113-123) and int16 gains
                 (python/intref.py:126-130)
  formats        per-layer (bits, f) of formats.json (Model.fmt, python/intref.py:154-160)
  tables         exp / SiLU / RoPE, 50-digit mpmath rounded half up (python/intref.py:66-108)
  layout         c/intref.c:8-13 (writer python/export_vectors.py:24-45)

Token windows: rng(1).integers(0, 49152, (4096, 512)); sequence w is row w, first T ids.
The bytes are identical to what the reference exporter writes for the same float weights (the
test suite checks the sha256 against the reference's own export).
"""
import json
import math
import multiprocessing as mpc
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
V, D, NL = 49152, 576, 30
SHAPES = (("q", 576, 576), ("k", 192, 576), ("v", 192, 576), ("o", 576, 576), ("gate", 1536, 576),
          ("up", 1536, 576), ("down", 576, 1536))
OUTLIER_CHANNELS = (7, 101, 333, 507)
WEIGHT_SEED, IDS_SEED, IDS_ROWS = 0, 1, 4096


def _formats():
    with open(os.path.join(HERE, "formats.json")) as f:
        j = json.load(f)
    return j["wide"], int(j["f_y"])


def _rows_int8(W):
    W = W.astype(np.float64)
    s = np.abs(W).max(1) / 127.0
    s = np.where(s == 0, 1.0, s)
    n = (13 - np.floor(np.log2(s))).astype(np.int64)
    m = np.rint(s * 2.0 ** n).astype(np.int64)
    if m.min() < 2 ** 13 or m.max() > 2 ** 14:
        raise ValueError("row multiplier outside [2^13, 2^14]")
    step = m * 2.0 ** (-n.astype(np.float64))
    return np.clip(np.rint(W / step[:, None]), -127, 127).astype(np.int8), m, n


def _gain_int16(w):
    w = w.astype(np.float64)
    f = 14 - int(math.floor(math.log2(np.abs(w).max())))
    return np.clip(np.rint(w * 2.0 ** f), -32768, 32767).astype(np.int64), f


def _mp():
    import mpmath
    return mpmath


def _half_up(mp, v):
    return int(mp.floor(v + mp.mpf(1) / 2))


def _exp_table():
    mp = _mp()
    with mp.workdps(50):
        one = mp.mpf(2) ** 30
        return np.array([_half_up(mp, one * mp.exp(-mp.mpf(d) / 128)) for d in range(1537)], dtype=np.int64)


def _silu(key):
    f_in, f_out, bits = key
    mp = _mp()
    vals = np.empty(65536, dtype=np.int64)
    with mp.workdps(50):
        step, scale = mp.mpf(2) ** (-f_in), mp.mpf(2) ** f_out
        for i in range(65536):
            x = (i - 32768) * step
            vals[i] = _half_up(mp, x / (1 + mp.exp(-x)) * scale)
    return key, np.clip(vals, -(1 << (bits - 1)), (1 << (bits - 1)) - 1)


def _rope(T=512):
    mp = _mp()
    C = np.empty((T, 32), dtype=np.int64)
    S = np.empty((T, 32), dtype=np.int64)
    with mp.workdps(50):
        inv = [mp.mpf(100000) ** (-mp.mpf(2 * j) / 64) for j in range(32)]
        one = mp.mpf(2) ** 30
        for p in range(T):
            for j in range(32):
                C[p, j] = _half_up(mp, mp.cos(p * inv[j]) * one)
                S[p, j] = _half_up(mp, mp.sin(p * inv[j]) * one)
    return C, S


def write_model_bin(path, seed=WEIGHT_SEED, outlier=False, procs=None):
    """Write the synthetic model.bin to `path` (about 154 MB).  SiLU tables are computed in a spawn
    pool (safe after CUDA initialisation)."""
    fms, f_y = _formats()
    keys = sorted({(fm[17], fm[21], fm[20]) for fm in fms})
    ctx = mpc.get_context("spawn")
    with ctx.Pool(min(len(keys), procs or os.cpu_count() or 1)) as pool:
        silu = dict(pool.map(_silu, keys))
    rng = np.random.default_rng(seed)
    sd = np.float32(0.02)
    gain = np.ones(D, dtype=np.float32)
    if outlier:
        gain[list(OUTLIER_CHANNELS)] = np.float32(50.0)
    gq, gf = _gain_int16(gain)
    tmp = path + ".partial"
    with open(tmp, "wb") as f:
        def w(a, dt):
            f.write(np.ascontiguousarray(a, dtype=dt).tobytes())
        q, m, n = _rows_int8(rng.standard_normal((V, D), dtype=np.float32) * sd)
        w(q, np.int8); w(m, np.int64); w(n, np.int64)
        w(gq, np.int64); w([gf], np.int64); w([f_y], np.int64)
        w(_exp_table(), np.int64)
        C, S = _rope()
        w(C, np.int64); w(S, np.int64)
        for l in range(NL):
            fm = fms[l]
            w(fm, np.int64)
            w(gq, np.int64); w([gf], np.int64)
            w(gq, np.int64); w([gf], np.int64)
            for _, N, K in SHAPES:
                q, m, n = _rows_int8(rng.standard_normal((N, K), dtype=np.float32) * sd)
                w(q, np.int8); w(m, np.int64); w(n, np.int64)
            w(silu[(fm[17], fm[21], fm[20])], np.int64)
    os.replace(tmp, path)
    return path


def token_table(rows=IDS_ROWS, seed=IDS_SEED):
    return np.random.default_rng(seed).integers(0, V, size=(rows, 512), dtype=np.int64)
