"""Drop-in replacement for the reference's python/intref.py module, backed by the B200 engine.

Put this package directory on sys.path where the reference's python/ directory was, and
`import intref` gives the same names (python/intref.py):

  Model(wide=True, proposal_path=None)   .forward(ids) .block(l, x) .embed(ids) .rmsnorm(...)
                                         .linear(...) .fmt(site, l), attributes L, cfg, emb_q,
                                         emb_m, emb_n, layers, final_gain, rope
  rs, sat, matmul_exact, exp_table, silu_table, rope_tables, dequant, F_RES, F_SCORE, ...

Differences a caller must know:
  * Weights come from a model.bin (the file python/export_vectors.py writes), not from the HF
    checkpoint: pass model_bin=... or set EII_MODEL_BIN.  The per-layer formats are the ones stored
    in model.bin (wide mode).  wide=False (narrow comparison mode) derives the INT16 formats of the
    flagged sites from them (f = 31 - k in wide mode, 15 - k in narrow mode) and regenerates the SiLU
    tables whose format changes, in memory (eii_table_silu).
  * forward(ids, narrow_residual=True) needs the k of the resid_in / resid_out sites: from the
    reference's scaling_proposal.json (proposal_path=...) or, by default, the format table shipped
    with this package (formats.json, derived from that file).
  * forward/block/embed/rmsnorm/linear run on the GPU through libeii.so; there is no CPU path.
  * block(l, x, trace=dict) fills the reference's per-site trace; rmsnorm(trace=...) raises
    NotImplementedError.
  * exp_table/silu_table/rope_tables return the tables of the most recently loaded model.bin
    (the reference regenerates them with mpmath; the engine, like c/intref.c, reads them).
  * rs, sat and dequant are the host-side numpy helpers of the reference's conventions.
"""
import os

import numpy as np

import _eii

F_RES = 15
F_SCORE = 7
DMAX = 12 * 128
EXP_BITS = 30
EPS_S = 6184753
R_ISQRT = 40
I64 = np.int64

V, D, NL = 49152, 576, 30
_LIN = (("q", 576, 576), ("k", 192, 576), ("v", 192, 576), ("o", 576, 576), ("gate", 1536, 576),
        ("up", 1536, 576), ("down", 576, 1536))
_SITES = ("norm1_out", "q_proj", "k_proj", "v_proj", "q_rope", "k_rope", "attn_ctx", "norm2_out", "gate_proj",
          "up_proj", "silu_gate", "mlp_gated")

_last_model = None


def rs(x, n):
    """Rounding right shift, ties toward +inf; n <= 0 is an exact left shift (python/intref.py:42-50)."""
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
    """Clip to the signed `bits` range (python/intref.py:53-55)."""
    return np.clip(x, -(1 << (bits - 1)), (1 << (bits - 1)) - 1)


def dequant(q, f):
    return q.astype(np.float64) * 2.0 ** (-f)


def _model():
    if _last_model is None:
        raise RuntimeError("no Model has been constructed yet (the engine reads tables and runs on a loaded model)")
    return _last_model


def matmul_exact(A, Wf, bound_a, wmax=127):
    """A int [T,K] @ W [N,K]^T, exact, on the GPU (python/intref.py:58-63).  W must hold int8 values,
    K a multiple of 32 up to 1536, N a multiple of 16, |A| < 2^31."""
    A = np.asarray(A, dtype=I64)
    W = np.asarray(Wf)
    if not (np.all(W == np.rint(W)) and W.min(initial=0) >= -128 and W.max(initial=0) <= 127):
        raise NotImplementedError("matmul_exact on the GPU needs int8-valued weights")
    bits_in = 16 if bound_a <= (1 << 15) else 32
    N = W.shape[0]
    ones = np.ones(N, dtype=I64)
    shifts = np.ones(N, dtype=I64)
    _, acc = _model()._eng.linear(A, bits_in, W.astype(np.int8), ones, shifts, 0, 0, 64)
    return acc


def exp_table():
    return _model()._exp


def silu_table(f_in, f_out, out_bits):
    m = _model()
    for l in range(m.L):
        F = m._fm[l]
        if (F[17], F[21], F[20]) == (f_in, f_out, out_bits):
            return m.layers[l]["silu"]
    raise KeyError(f"no layer of the loaded model uses SiLU table {(f_in, f_out, out_bits)}")


def rope_tables(T):
    m = _model()
    if T > 512:
        raise ValueError("RoPE tables cover positions < 512")
    return m.rope[0][:T], m.rope[1][:T]


class Model:
    def __init__(self, wide=True, proposal_path=None, model_bin=None, device=0):
        global _last_model
        path = model_bin or os.environ.get("EII_MODEL_BIN")
        if not path:
            raise ValueError("pass model_bin= or set EII_MODEL_BIN to a model.bin written by export_vectors.py")
        with open(path, "rb") as f:
            buf = f.read()
        self._parse(buf)
        if not wide:
            buf = self._narrow(buf)
            self._parse(buf)
        self._proposal_path = proposal_path
        self._eng = _eii.Engine(np.frombuffer(buf, dtype=np.uint8), device)
        self.wide = bool(wide)
        self.cfg = {"num_hidden_layers": NL}
        self.L = NL
        _last_model = self

    def _parse(self, buf):
        off = 0

        def take(count, dt):
            nonlocal off
            a = np.frombuffer(buf, dtype=dt, count=count, offset=off)
            off += a.nbytes
            return a
        self.emb_q = take(V * D, np.int8).reshape(V, D).astype(np.float64)
        self.emb_m, self.emb_n = take(V, I64), take(V, I64)
        fq = take(D, I64)
        ff = int(take(1, I64)[0])
        self.final_gain = (fq, ff)
        self.f_y = int(take(1, I64)[0])
        self._exp = take(DMAX + 1, I64)
        self.rope = (take(512 * 32, I64).reshape(512, 32), take(512 * 32, I64).reshape(512, 32))
        self.layers, self._fm, self._fm_off, self._silu_off = [], [], [], []
        for _ in range(NL):
            self._fm_off.append(off)
            fm = [int(v) for v in take(24, I64)]
            d = {"ln1": (take(D, I64), int(take(1, I64)[0])), "ln2": (take(D, I64), int(take(1, I64)[0]))}
            for nm, N, K in _LIN:
                d[nm] = (take(N * K, np.int8).reshape(N, K).astype(np.float64), take(N, I64), take(N, I64))
            self._silu_off.append(off)
            d["silu"] = take(65536, I64)
            self.layers.append(d)
            self._fm.append(fm)
        if off != len(buf):
            raise ValueError("model.bin size does not match the layout of c/intref.c:8-13")

    def _narrow(self, buf):
        """The model.bin of the narrow comparison mode (python/intref.py:152-160): every INT32 site
        (f = 31 - k) becomes INT16 with f = 15 - k, and the SiLU tables whose (f_g, f_s, bits_s)
        change are regenerated (eii_table_silu, python/intref.py:81-94)."""
        out = bytearray(buf)
        cache = {}
        for l in range(NL):
            fm = self._fm[l]
            new = list(fm)
            for i in range(0, 24, 2):
                if fm[i] == 32:
                    new[i], new[i + 1] = 16, fm[i + 1] - 16
            out[self._fm_off[l]:self._fm_off[l] + 24 * 8] = np.asarray(new, dtype=I64).tobytes()
            gi, si = _SITES.index("gate_proj"), _SITES.index("silu_gate")
            old_key = (fm[2 * gi + 1], fm[2 * si + 1], fm[2 * si])
            key = (new[2 * gi + 1], new[2 * si + 1], new[2 * si])
            if key != old_key:
                if key not in cache:
                    cache[key] = _eii.table_silu(*key)
                out[self._silu_off[l]:self._silu_off[l] + 65536 * 8] = np.asarray(cache[key], dtype=I64).tobytes()
        return bytes(out)

    def _resid_k(self):
        """k of the resid_in|l and resid_out|l sites (the narrow residual grid)."""
        import json
        if self._proposal_path:
            with open(self._proposal_path) as f:
                sites = json.load(f)["sites"]
            return ([int(sites[f"resid_in|{l}"]["k"]) for l in range(NL)],
                    [int(sites[f"resid_out|{l}"]["k"]) for l in range(NL)])
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "formats.json")) as f:
            rk = json.load(f)["resid_k"]
        return [int(v) for v in rk["resid_in"]], [int(v) for v in rk["resid_out"]]

    def fmt(self, site, l):
        """(bits, f) of a site at layer l, as stored in model.bin (python/intref.py:154-160)."""
        if site == "final_out" and l == NL:
            return 16, self.f_y
        i = _SITES.index(site)
        fm = self._fm[l]
        return fm[2 * i], fm[2 * i + 1]

    def embed(self, ids):
        return self._eng.embed(np.asarray(ids, dtype=I64))

    def rmsnorm(self, x, gain, f_out, bits_out, trace=None, tag=""):
        if trace is not None:
            raise NotImplementedError("per-site trace is not implemented by the B200 engine yet")
        wq, fw = gain
        return self._eng.rmsnorm(x, wq, fw, f_out, bits_out)

    def linear(self, a, bound_a, W, f_in, f_out, bits_out):
        q, m, n = W
        bits_in = 16 if bound_a <= (1 << 15) else 32
        out, acc = self._eng.linear(np.asarray(a, dtype=I64), bits_in, np.asarray(q).astype(np.int8), m, n,
                                    f_in, f_out, bits_out)
        return out, acc

    def block(self, l, x, trace=None):
        """Model.block (python/intref.py:192-286); with a trace dict, every site and the "_f" exponents."""
        x = np.asarray(x, dtype=I64)
        if trace is None:
            return self._eng.block(l, x, T=x.shape[0])
        out, sites = self._eng.block_trace(l, x)
        trace.update(sites)
        f = {k: self.fmt(k, l)[1] for k in ("norm1_out", "q_proj", "k_proj", "v_proj", "q_rope", "k_rope", "attn_ctx",
                                             "norm2_out", "gate_proj", "up_proj", "silu_gate")}
        bits_m, f_m0 = self.fmt("mlp_gated", l)
        f["mlp_gated"] = min(f_m0, f["silu_gate"] + f["up_proj"]) if bits_m == 32 else f_m0  # python/intref.py:274
        trace["_f"] = {"resid_in": F_RES, "o_res": F_RES, "resid_mid": F_RES, "down_res": F_RES, "resid_out": F_RES,
                       "attn_score": F_SCORE, "attn_prob": 16, **f}
        return out

    def forward(self, ids, narrow_residual=False):
        """python/intref.py:288-301; narrow_residual puts the residual on its INT16 grid before and
        after every layer (python/intref.py:303-308), on the GPU (eii_set_residual_grid)."""
        if narrow_residual:
            k_in, k_out = self._resid_k()
            self._eng.set_residual_grid(k_in, k_out)
        try:
            x = self.embed(ids)
            for l in range(self.L):
                x = self.block(l, x)
            return self._eng.logits(x)
        finally:
            if narrow_residual:
                self._eng.set_residual_grid(None, None)

    def close(self):
        self._eng.close()
