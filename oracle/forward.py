"""Numpy restatement of the reference's integer forward pass (TEST INFRASTRUCTURE: oracle only).

Follows python/intref.py (the definition) step by step, reading every weight, format and table
from a parsed model.bin, as c/intref.c does.  Matrix products are exact: int64 operands are
widened to float64 for BLAS only when every partial sum stays below 2^53 (asserted, as
intref.py:61,247 do); otherwise they are split into exact 16-bit halves first.

  rs, sat            intref.py:42-55
  embed              intref.py:163-166
  rmsnorm            intref.py:168-184      (exact 128-bit total via Python ints)
  linear             intref.py:186-190
  block              intref.py:192-286      (RoPE :212-225, attention :227-254, o :256-261,
                                             MLP :264-281)
  final norm+logits  intref.py:296-300
  forward            intref.py:288-301

Sequences are independent: block_batch runs the linears on all rows of a batch of equal-length
sequences at once and attention per sequence, which gives the same integers as running
intref.Model.forward on each sequence.
"""
import math

import numpy as np

F_RES = 15
F_SCORE = 7
DMAX = 12 * 128
EPS_S = 6184753
R_ISQRT = 40
NH, NKV, HD = 9, 3, 64
I64 = np.int64


def rs(x, n):
    """Rounding right shift, ties toward +inf; n <= 0 is an exact left shift (intref.py:42-50)."""
    if np.isscalar(n):
        n = int(n)
        if n <= 0:
            return np.asarray(x, dtype=I64) << (-n)
        return (np.asarray(x, dtype=I64) + (I64(1) << (n - 1))) >> n
    n = np.asarray(n, dtype=I64)
    if not (n >= 1).all():
        raise AssertionError("per-element shift must be >= 1")
    return (np.asarray(x, dtype=I64) + (I64(1) << (n - 1))) >> n


def sat(x, bits):
    """Clip to signed `bits` (intref.py:53-55); bits >= 64 is the identity (c/intref.c:33-37)."""
    if bits >= 64:
        return x
    return np.clip(x, -(1 << (bits - 1)), (1 << (bits - 1)) - 1)


def matmul_exact(A, W, bound_a, wmax=127):
    """int64 A [M,K] @ int W [N,K]^T, exact.  float64 BLAS when the 2^53 bound holds
    (intref.py:58-63), else A is split into 16-bit halves that each satisfy it."""
    A = np.asarray(A, dtype=I64)
    K = A.shape[1]
    Wf = np.asarray(W, dtype=np.float64)
    if bound_a * wmax * K < 2.0 ** 53:
        return np.rint(A.astype(np.float64) @ Wf.T).astype(I64)
    hi = A >> 16
    lo = A & 0xFFFF
    assert (1 << 16) * wmax * K < 2.0 ** 53 and (bound_a >> 16) * wmax * K < 2.0 ** 53
    return (np.rint(hi.astype(np.float64) @ Wf.T).astype(I64) << 16) + \
        np.rint(lo.astype(np.float64) @ Wf.T).astype(I64)


def fm_unpack(fm):
    fm = [int(v) for v in fm]
    keys = ("h", "q", "k", "v", "qr", "kr", "c", "h2", "g", "u", "s", "m")
    return {k: (fm[2 * i], fm[2 * i + 1]) for i, k in enumerate(keys)}


def embed(mdl, ids):
    # intref.py:163-166
    ids = np.asarray(ids, dtype=I64).reshape(-1)
    q = mdl["emb_q"][ids].astype(I64)
    x = q * mdl["emb_m"][ids][:, None]
    return rs(x, (mdl["emb_n"][ids] - F_RES)[:, None])


def isqrt_recip(S_plus_eps):
    """U = isqrt(floor(2^80 / T)) for a Python int T (intref.py:177)."""
    return math.isqrt((1 << (2 * R_ISQRT)) // S_plus_eps)


def rmsnorm_U(x):
    """Per-row U of intref.py:170-177 (exact 128-bit total S + eps)."""
    hi = x >> 16
    lo = x & 0xFFFF
    A = (hi * hi).sum(1)
    B = (hi * lo).sum(1)
    C = (lo * lo).sum(1)
    U = np.empty(x.shape[0], dtype=I64)
    for t in range(x.shape[0]):
        S = (int(A[t]) << 32) + (int(B[t]) << 17) + int(C[t])
        U[t] = isqrt_recip(S + EPS_S)
    return U


def rmsnorm(x, gain_q, gain_f, f_out, bits_out, trace=None, tag=""):
    # intref.py:168-184
    x = np.asarray(x, dtype=I64)
    U = rmsnorm_U(x)
    z = rs(x * U[:, None], 16)
    acc = z * np.asarray(gain_q, dtype=I64)[None, :] * 3
    out = sat(rs(acc, 21 + int(gain_f) - f_out), bits_out)
    if trace is not None:
        trace[tag + "_U"] = U
        trace[tag + "_z"] = z
        trace[tag + "_out"] = out
    return out


def linear(a, bound_a, W, f_in, f_out, bits_out):
    # intref.py:186-190
    q, m, n = W
    acc = matmul_exact(a, q, bound_a)
    assert np.abs(acc).max(initial=0) * int(m.max()) < 2 ** 63
    return sat(rs(acc * m[None, :], n + f_in - f_out), bits_out), acc


def rope(a, C, S, nheads, f_in, f_o, bits_o):
    # intref.py:212-222; a [T, nheads*64], C/S [T, 32]
    T = a.shape[0]
    a = a.reshape(T, nheads, HD)
    a1, a2 = a[:, :, :32], a[:, :, 32:]
    c, s = C[:, None, :], S[:, None, :]
    o = np.concatenate([a1 * c - a2 * s, a2 * c + a1 * s], axis=2)
    return sat(rs(o, 30 + f_in - f_o), bits_o)


def attention(qr, kr, v, E, f_qr, f_kr, f_v, f_c, bits_c, bits_qr, bits_kr, bits_v, trace=None):
    """One sequence: qr [T,9,64], kr/v [T,3,64] -> ctx [T,576]  (intref.py:227-254)."""
    T = qr.shape[0]
    bq, bk, bv = 1 << (bits_qr - 1), 1 << (bits_kr - 1), 1 << (bits_v - 1)
    shift_s = f_qr + f_kr + 3 - F_SCORE
    assert shift_s >= 1
    causal = np.tril(np.ones((T, T), dtype=bool))
    ctx = np.empty((T, NH, HD), dtype=I64)
    sc_all, p_all = [], []
    for hh in range(NH):
        g = hh // 3
        acc = matmul_exact(qr[:, hh, :], kr[:, g, :], bq, wmax=bk)
        s = sat(rs(acc, shift_s), 16)
        s_m = np.where(causal, s, -(1 << 40))
        rowmax = s_m.max(1, keepdims=True)
        d = rowmax - s
        valid = causal & (d <= DMAX)
        e = np.where(valid, E[np.clip(d, 0, DMAX)], 0)
        Z = e.sum(1, keepdims=True)
        P = (e * 65536 + Z // 2) // Z
        assert 65536 * bv * T < 2 ** 53
        acc2 = np.rint(P.astype(np.float64) @ v[:, g, :].astype(np.float64)).astype(I64)
        ctx[:, hh, :] = sat(rs(acc2, 16 + f_v - f_c), bits_c)
        if trace is not None:
            sc_all.append(np.where(causal, s, 0))
            p_all.append(P)
    if trace is not None:
        trace["attn_score"] = np.stack(sc_all)
        trace["attn_prob"] = np.stack(p_all)
        trace["attn_ctx"] = ctx.reshape(T, -1)
    return ctx.reshape(T, NH * HD)


def block_batch(mdl, l, x, T, trace=None):
    """Layer l on x [n_seq*T, 576] (sequence-major rows) -> new residual (intref.py:192-286)."""
    Ly = mdl["layers"][l]
    F = fm_unpack(Ly["fm"])
    M = x.shape[0]
    assert M % T == 0
    nseq = M // T
    if trace is not None:
        trace["resid_in"] = x.copy()
    bits_h, f_h = F["h"]
    h = rmsnorm(x, Ly["ln1_q"], Ly["ln1_f"], f_h, bits_h, trace, "norm1")
    bh = 1 << (bits_h - 1)
    (bits_q, f_q), (bits_k, f_k), (bits_v, f_v) = F["q"], F["k"], F["v"]
    q, _ = linear(h, bh, Ly["q"], f_h, f_q, bits_q)
    k, _ = linear(h, bh, Ly["k"], f_h, f_k, bits_k)
    v, _ = linear(h, bh, Ly["v"], f_h, f_v, bits_v)
    (bits_qr, f_qr), (bits_kr, f_kr) = F["qr"], F["kr"]
    bits_c, f_c = F["c"]
    C, S = mdl["rope_c"][:T].astype(I64), mdl["rope_s"][:T].astype(I64)
    ctx = np.empty((M, NH * HD), dtype=I64)
    qr_all, kr_all = [], []
    for sidx in range(nseq):
        r = slice(sidx * T, (sidx + 1) * T)
        qr = rope(q[r], C, S, NH, f_q, f_qr, bits_qr)
        kr = rope(k[r], C, S, NKV, f_k, f_kr, bits_kr)
        if trace is not None:
            qr_all.append(qr.reshape(T, -1)); kr_all.append(kr.reshape(T, -1))
        ctx[r] = attention(qr, kr, v[r].reshape(T, NKV, HD), mdl["exp"], f_qr, f_kr, f_v, f_c,
                           bits_c, bits_qr, bits_kr, bits_v, trace if nseq == 1 else None)
    if trace is not None:
        trace.update(q_proj=q, k_proj=k, v_proj=v, q_rope=np.concatenate(qr_all),
                     k_rope=np.concatenate(kr_all))
        if nseq != 1:
            trace["attn_ctx"] = ctx
    q_o, m_o, n_o = Ly["o"]
    acc = matmul_exact(ctx, q_o, 1 << (bits_c - 1))
    assert np.abs(acc).max(initial=0) * int(m_o.max()) < 2 ** 63
    o_res = rs(acc * m_o[None, :], n_o + f_c - F_RES)
    x = sat(x + o_res, 32)
    if trace is not None:
        trace["o_res"] = o_res; trace["resid_mid"] = x.copy()
    bits_h2, f_h2 = F["h2"]
    h2 = rmsnorm(x, Ly["ln2_q"], Ly["ln2_f"], f_h2, bits_h2, trace, "norm2")
    bh2 = 1 << (bits_h2 - 1)
    (bits_g, f_g), (bits_u, f_u) = F["g"], F["u"]
    g_, _ = linear(h2, bh2, Ly["gate"], f_h2, f_g, bits_g)
    u_, _ = linear(h2, bh2, Ly["up"], f_h2, f_u, bits_u)
    bits_s, f_s = F["s"]
    sg = np.asarray(Ly["silu"], dtype=I64)[g_ + 32768]
    bits_m, f_m0 = F["m"]
    f_m = min(f_m0, f_s + f_u) if bits_m == 32 else f_m0
    gated = sat(rs(sg * u_, f_s + f_u - f_m), bits_m)
    if trace is not None:
        trace.update(gate_proj=g_, up_proj=u_, silu_gate=sg, mlp_gated=gated)
    q_d, m_d, n_d = Ly["down"]
    acc = matmul_exact(gated, q_d, 1 << (bits_m - 1))
    assert np.abs(acc).max(initial=0) * int(m_d.max()) < 2 ** 63
    d_res = rs(acc * m_d[None, :], n_d + f_m - F_RES)
    x = sat(x + d_res, 32)
    if trace is not None:
        trace["down_res"] = d_res; trace["resid_out"] = x.copy()
        trace["_f"] = {"resid_in": F_RES, "o_res": F_RES, "resid_mid": F_RES, "down_res": F_RES,
                       "resid_out": F_RES, "attn_score": F_SCORE, "attn_prob": 16,
                       "norm1_out": f_h, "q_proj": f_q, "k_proj": f_k, "v_proj": f_v,
                       "q_rope": f_qr, "k_rope": f_kr, "attn_ctx": f_c, "norm2_out": f_h2,
                       "gate_proj": f_g, "up_proj": f_u, "silu_gate": f_s, "mlp_gated": f_m}
    return x


def final_norm(mdl, x):
    # intref.py:296-297; f_y comes from model.bin
    return rmsnorm(x, mdl["final_q"], mdl["final_f"], mdl["f_y"], 16)


def logits_from_y(mdl, y):
    # intref.py:298-300
    acc = matmul_exact(y, mdl["emb_q"], 1 << 15)
    return rs(acc * mdl["emb_m"][None, :], mdl["emb_n"] + mdl["f_y"] - 16)


def forward(mdl, ids, want_states=True, layers=None):
    """ids [T] or [n_seq, T] -> dict(embed [n_seq,T,576], resid [L,n_seq,T,576], logits
    [n_seq,T,V]) as int64.  The per-layer residuals are the checkpoints export_vectors.py
    writes (python/export_vectors.py:47-57)."""
    ids = np.asarray(ids, dtype=I64)
    if ids.ndim == 1:
        ids = ids[None, :]
    nseq, T = ids.shape
    L = len(mdl["layers"]) if layers is None else layers
    x = embed(mdl, ids)
    out = {"embed": x.reshape(nseq, T, -1).copy()}
    res = []
    for l in range(L):
        x = block_batch(mdl, l, x, T)
        if want_states:
            res.append(x.reshape(nseq, T, -1).copy())
    if want_states:
        out["resid"] = np.stack(res) if res else np.zeros((0, nseq, T, 576), dtype=I64)
    y = final_norm(mdl, x)
    out["logits"] = logits_from_y(mdl, y).reshape(nseq, T, -1)
    return out
