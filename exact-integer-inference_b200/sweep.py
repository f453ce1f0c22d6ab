"""Workload definition of the stand-alone contraction sweep (Model.linear, python/intref.py:186-190).

Four weight shapes of the seeded synthetic model, each at M = 512 ... 262144 activation rows:

  q_576x576         layer 0 q        norm1_out|0  (INT16)  -> q_proj|0 format  (SAT16)
  gate_1536x576     layer 11 gate    norm2_out|11 (INT16)  -> gate_proj|11 format (SAT16)
  down_576x1536     layer 0 down     mlp_gated|0  (INT32)  -> residual grid f = 15, SAT32
  logits_49152x576  tied embedding   final_out|30 (INT16)  -> f = 16, SAT32 (the logits of
                                                              python/intref.py:298-300 fit int32)

Activations are int32 values drawn uniform over the full signed range of the input format, in
blocks of 4096 rows: block b of case c at M rows comes from np.random.default_rng([SEED, c, M, b]);
row 0 is all -2^(bits-1) and row 1 all 2^(bits-1) - 1.  The same generator feeds the golden
digests (tests/golden/make_golden.py runs the reference's own Model.linear on it), the GPU tests
and bench.py.

Digests (mod 2^64), per row r of an [M, N] result, with mix64 the weight function of the logits
digest (include/eii.h):
    D_out[r] = sum_c uint32(out[r, c]) * mix64(2^32 + c)
    D_acc[r] = sum_c uint64(acc[r, c]) * mix64(2^32 + c)        (acc the exact int64 contraction)
and per 4096-row block b:  B[b] = sum_{r in b} D[r] * mix64(r);  the case digest is sum_b B[b].
eii_linear_plan_run produces D_out and D_acc on the device.
"""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SEED = 20260005
BLOCK = 4096
MS = (512, 4096, 32768, 262144)
V, D, NL = 49152, 576, 30
_SITES = ("norm1_out", "q_proj", "k_proj", "v_proj", "q_rope", "k_rope", "attn_ctx", "norm2_out", "gate_proj",
          "up_proj", "silu_gate", "mlp_gated")
_LIN = (("q", 576, 576), ("k", 192, 576), ("v", 192, 576), ("o", 576, 576), ("gate", 1536, 576),
        ("up", 1536, 576), ("down", 576, 1536))

# name, weight (matrix, layer), input site (site, layer), output (site, layer) or ("grid", f_out, bits_out)
CASES = (
    ("q_576x576", ("q", 0), ("norm1_out", 0), ("q_proj", 0)),
    ("gate_1536x576", ("gate", 11), ("norm2_out", 11), ("gate_proj", 11)),
    ("down_576x1536", ("down", 0), ("mlp_gated", 0), ("grid", 15, 32)),
    ("logits_49152x576", ("embed", None), ("final_out", 30), ("grid", 16, 32)),
)


def _formats():
    with open(os.path.join(HERE, "formats.json")) as f:
        j = json.load(f)
    return j["wide"], int(j["f_y"])


def case_formats(ci):
    """(bits_in, f_in, f_out, bits_out) of case ci, from the wide format table (Model.fmt,
    python/intref.py:154-160) of the synthetic model."""
    wide, f_y = _formats()
    _, _, (si, li), out = CASES[ci]
    if si == "final_out":
        bits_in, f_in = 16, f_y
    else:
        k = _SITES.index(si)
        bits_in, f_in = wide[li][2 * k], wide[li][2 * k + 1]
    if out[0] == "grid":
        f_out, bits_out = out[1], out[2]
    else:
        k = _SITES.index(out[0])
        bits_out, f_out = wide[out[1]][2 * k], wide[out[1]][2 * k + 1]
    return bits_in, f_in, f_out, bits_out


def weights(model_bin, ci):
    """(W int8 [N, K], m int64 [N], n int64 [N]) of case ci from a model.bin (layout c/intref.c:8-13)."""
    buf = model_bin if isinstance(model_bin, (bytes, bytearray, memoryview)) else open(model_bin, "rb").read()
    wname, wl = CASES[ci][1]
    if wname == "embed":
        q = np.frombuffer(buf, np.int8, V * D, 0).reshape(V, D)
        m = np.frombuffer(buf, np.int64, V, V * D)
        n = np.frombuffer(buf, np.int64, V, V * D + 8 * V)
        return q, m, n
    off = V * D + 16 * V + 8 * D + 16 + 8 * (12 * 128 + 1) + 2 * 8 * 512 * 32
    per = 24 * 8 + 2 * (8 * D + 8) + sum(N * K + 16 * N for _, N, K in _LIN) + 65536 * 8
    off += wl * per + 24 * 8 + 2 * (8 * D + 8)
    for name, N, K in _LIN:
        if name == wname:
            q = np.frombuffer(buf, np.int8, N * K, off).reshape(N, K)
            m = np.frombuffer(buf, np.int64, N, off + N * K)
            n = np.frombuffer(buf, np.int64, N, off + N * K + 8 * N)
            return q, m, n
        off += N * K + 16 * N
    raise KeyError(wname)


def blocks(M):
    return (M + BLOCK - 1) // BLOCK


def activation_block(ci, M, b, K, bits):
    """Rows [4096 b, min(4096 (b + 1), M)) of case ci's int32 activations at M rows."""
    rows = min(BLOCK, M - BLOCK * b)
    rng = np.random.default_rng([SEED, ci, M, b])
    a = rng.integers(-(1 << (bits - 1)), 1 << (bits - 1), size=(rows, K), dtype=np.int32)
    if b == 0:
        a[0] = -(1 << (bits - 1))
        a[1] = (1 << (bits - 1)) - 1
    return a


def mix64(z):
    M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z + np.uint64(0x9E3779B97F4A7C15)) & M64
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return (z ^ (z >> np.uint64(31))) | np.uint64(1)


def col_weights(N):
    return mix64(np.arange(N, dtype=np.uint64) + np.uint64(1 << 32))


def row_digests(x, N, as_u32):
    """Per-row digests of an [rows, N] integer array: sum_c u(x[r, c]) * mix64(2^32 + c) mod 2^64,
    u = uint32 of the value (as_u32) or its two's-complement uint64."""
    x = np.asarray(x)
    u = x.astype(np.int64).astype(np.uint32).astype(np.uint64) if as_u32 else x.astype(np.int64).view(np.uint64)
    with np.errstate(over="ignore"):
        return (u * col_weights(N)[None, :]).sum(axis=1, dtype=np.uint64)


def block_digests(row_dig, M):
    """B[b] = sum over the rows r of block b of row_dig[r] * mix64(r), for all blocks of M rows."""
    row_dig = np.asarray(row_dig, dtype=np.uint64)
    w = mix64(np.arange(M, dtype=np.uint64))
    out = []
    with np.errstate(over="ignore"):
        for b in range(blocks(M)):
            s = slice(BLOCK * b, min(BLOCK * (b + 1), M))
            out.append(int((row_dig[s] * w[s]).sum(dtype=np.uint64)))
    return out


def total(blocks_):
    return sum(blocks_) % (1 << 64)


def hexes(vals):
    return [f"{v:016x}" for v in vals]
