"""model.bin reader/writer (TEST INFRASTRUCTURE: oracle only).

Layout, little endian, sequential (c/intref.c:8-13; writer python/export_vectors.py:24-45):
  emb_q int8[V*D], emb_m i64[V], emb_n i64[V], final_gain_q i64[D], final_gain_f i64, f_y i64,
  exp_table i64[DMAX+1], rope_cos i64[512*32], rope_sin i64[512*32],
  per layer: fmt i64[24] (bits,f pairs of norm1_out q_proj k_proj v_proj q_rope k_rope attn_ctx
             norm2_out gate_proj up_proj silu_gate mlp_gated), ln1_q i64[D], ln1_f i64,
             ln2_q i64[D], ln2_f i64, then q,k,v,o,gate,up,down each as int8[N*K], m i64[N],
             n i64[N], then silu table i64[65536].
"""
import numpy as np

V, D, DFF, NL = 49152, 576, 1536, 30
DMAX = 12 * 128
ROPE_POS = 512
LIN_NAMES = ("q", "k", "v", "o", "gate", "up", "down")
LIN_SHAPES = {"q": (576, 576), "k": (192, 576), "v": (192, 576), "o": (576, 576),
              "gate": (1536, 576), "up": (1536, 576), "down": (576, 1536)}
FMT_SITES = ("norm1_out", "q_proj", "k_proj", "v_proj", "q_rope", "k_rope", "attn_ctx",
             "norm2_out", "gate_proj", "up_proj", "silu_gate", "mlp_gated")


def model_bin_size():
    n = V * D + 2 * V * 8 + D * 8 + 16 + (DMAX + 1) * 8 + 2 * ROPE_POS * 32 * 8
    per = 24 * 8 + 2 * (D * 8 + 8) + 65536 * 8
    for nm in LIN_NAMES:
        N, K = LIN_SHAPES[nm]
        per += N * K + 2 * N * 8
    return n + NL * per


def write_model_bin(path, mdl):
    """mdl: dict with emb_q int8[V,D], emb_m, emb_n i64[V], final_q i64[D], final_f, f_y,
    exp i64[1537], rope_c, rope_s i64[512,32], layers: list of dicts (fm i64[24], ln1_q, ln1_f,
    ln2_q, ln2_f, <lin>: (q int8[N,K], m i64[N], n i64[N]), silu i64[65536])."""
    def w(f, a, dt):
        f.write(np.ascontiguousarray(a, dtype=dt).tobytes())
    with open(path, "wb") as f:
        w(f, mdl["emb_q"], np.int8); w(f, mdl["emb_m"], np.int64); w(f, mdl["emb_n"], np.int64)
        w(f, mdl["final_q"], np.int64); w(f, [mdl["final_f"]], np.int64); w(f, [mdl["f_y"]], np.int64)
        w(f, mdl["exp"], np.int64)
        w(f, mdl["rope_c"][:ROPE_POS], np.int64); w(f, mdl["rope_s"][:ROPE_POS], np.int64)
        for Ly in mdl["layers"]:
            w(f, Ly["fm"], np.int64)
            w(f, Ly["ln1_q"], np.int64); w(f, [Ly["ln1_f"]], np.int64)
            w(f, Ly["ln2_q"], np.int64); w(f, [Ly["ln2_f"]], np.int64)
            for nm in LIN_NAMES:
                q, m, n = Ly[nm]
                w(f, q, np.int8); w(f, m, np.int64); w(f, n, np.int64)
            w(f, Ly["silu"], np.int64)


def parse_model_bin(buf):
    """bytes-like of exactly model_bin_size() bytes -> dict in the write_model_bin shape."""
    buf = memoryview(buf)
    if len(buf) != model_bin_size():
        raise ValueError(f"model.bin has {len(buf)} bytes, expected {model_bin_size()}")
    off = [0]

    def take(count, dt, shape=None):
        nbytes = count * np.dtype(dt).itemsize
        a = np.frombuffer(buf[off[0]:off[0] + nbytes], dtype=dt)
        off[0] += nbytes
        return a.reshape(shape) if shape else a

    mdl = {"emb_q": take(V * D, np.int8, (V, D)), "emb_m": take(V, np.int64), "emb_n": take(V, np.int64)}
    mdl["final_q"] = take(D, np.int64)
    mdl["final_f"] = int(take(1, np.int64)[0])
    mdl["f_y"] = int(take(1, np.int64)[0])
    mdl["exp"] = take(DMAX + 1, np.int64)
    mdl["rope_c"] = take(ROPE_POS * 32, np.int64, (ROPE_POS, 32))
    mdl["rope_s"] = take(ROPE_POS * 32, np.int64, (ROPE_POS, 32))
    layers = []
    for _ in range(NL):
        Ly = {"fm": take(24, np.int64)}
        Ly["ln1_q"] = take(D, np.int64); Ly["ln1_f"] = int(take(1, np.int64)[0])
        Ly["ln2_q"] = take(D, np.int64); Ly["ln2_f"] = int(take(1, np.int64)[0])
        for nm in LIN_NAMES:
            N, K = LIN_SHAPES[nm]
            Ly[nm] = (take(N * K, np.int8, (N, K)), take(N, np.int64), take(N, np.int64))
        Ly["silu"] = take(65536, np.int64)
        layers.append(Ly)
    mdl["layers"] = layers
    assert off[0] == len(buf)
    return mdl


def read_model_bin(path):
    with open(path, "rb") as f:
        return parse_model_bin(f.read())
