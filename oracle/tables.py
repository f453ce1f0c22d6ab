"""Exact lookup tables of the integer semantics (TEST INFRASTRUCTURE: oracle only).

Restates python/intref.py:66-108 of the reference: every entry is a 50-digit
mpmath value rounded half up (floor(v + 1/2)).

  exp_table()               intref.py:73-77   2^30 * exp(-d/128), d = 0..1536
  silu_table(f_in, f_out,b) intref.py:81-93   SAT_b(round(silu(q 2^-f_in) 2^f_out)), q = -32768..32767
  rope_tables(T)            intref.py:97-108  round(cos/sin(p theta^(-2j/64)) 2^30), p < T, j < 32

The engine never regenerates these: it reads them from model.bin, exactly as
c/intref.c and cuda/intref.cu do.  The SiLU tables are the slow part (about
1.5 s each); silu_tables_parallel() spreads distinct tables over a spawn pool.
"""
import multiprocessing as mpc

import mpmath as mp
import numpy as np

EXP_BITS = 30
DMAX = 12 * 128
ROPE_THETA = 100000
HEAD_DIM = 64
ROPE_POS = 512


def _half_up(v):
    # intref.py:68-69
    return int(mp.floor(v + mp.mpf(1) / 2))


def exp_table():
    with mp.workdps(50):
        scale = mp.mpf(2) ** EXP_BITS
        return np.array([_half_up(scale * mp.exp(-mp.mpf(d) / 128)) for d in range(DMAX + 1)],
                        dtype=np.int64)


def silu_table(f_in, f_out, out_bits):
    with mp.workdps(50):
        step = mp.mpf(2) ** (-f_in)
        scale = mp.mpf(2) ** f_out
        vals = np.empty(65536, dtype=np.int64)
        for i in range(65536):
            x = (i - 32768) * step
            vals[i] = _half_up(x / (1 + mp.exp(-x)) * scale)
    lo, hi = -(1 << (out_bits - 1)), (1 << (out_bits - 1)) - 1
    return np.clip(vals, lo, hi)


def _silu_job(key):
    return key, silu_table(*key)


def silu_tables_parallel(keys, procs=None):
    """Distinct (f_in, f_out, bits) keys -> {key: table}.  Uses a spawn pool so it
    is safe to call after CUDA has been initialised in the parent."""
    keys = sorted(set(keys))
    if len(keys) <= 1 or procs == 1:
        return dict(_silu_job(k) for k in keys)
    ctx = mpc.get_context("spawn")
    with ctx.Pool(min(len(keys), procs or mpc.cpu_count())) as pool:
        return dict(pool.map(_silu_job, keys))


def rope_tables(T=ROPE_POS, theta=ROPE_THETA, head_dim=HEAD_DIM):
    half = head_dim // 2
    C = np.empty((T, half), dtype=np.int64)
    S = np.empty((T, half), dtype=np.int64)
    with mp.workdps(50):
        inv = [mp.mpf(theta) ** (-mp.mpf(2 * j) / head_dim) for j in range(half)]
        one30 = mp.mpf(2) ** 30
        for p in range(T):
            for j in range(half):
                a = p * inv[j]
                C[p, j] = _half_up(mp.cos(a) * one30)
                S[p, j] = _half_up(mp.sin(a) * one30)
    return C, S
