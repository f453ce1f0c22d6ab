"""ctypes binding of libeii.so (the C ABI of include/eii.h).

The shared library is built in-tree by build.py.  There is no fallback: if the library or a CUDA
device is missing, calls raise EiiError.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libeii.so")

EII_OK, EII_ERR_ARG, EII_ERR_IO, EII_ERR_CUDA, EII_ERR_DEVICE, EII_ERR_FORMAT = range(6)
STATUS_NAMES = {0: "EII_OK", 1: "EII_ERR_ARG", 2: "EII_ERR_IO", 3: "EII_ERR_CUDA", 4: "EII_ERR_DEVICE",
                5: "EII_ERR_FORMAT"}

VOCAB, D_MODEL, N_LAYERS = 49152, 576, 30
NUM_KERNEL_KINDS = 12


class EiiError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


_lib = None

_P = ctypes.c_void_p
_SIGS = {
    "eii_last_error": ([], ctypes.c_char_p),
    "eii_version": ([], ctypes.c_int),
    "eii_open": ([ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(_P)], ctypes.c_int),
    "eii_open_memory": ([_P, ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(_P)], ctypes.c_int),
    "eii_close": ([_P], None),
    "eii_forward": ([_P, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P, _P], ctypes.c_int),
    "eii_forward_device": ([_P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int64, _P, _P], ctypes.c_int),
    "eii_embed": ([_P, _P, ctypes.c_int, _P], ctypes.c_int),
    "eii_block": ([_P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, _P], ctypes.c_int),
    "eii_rmsnorm": ([_P, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P], ctypes.c_int),
    "eii_logits": ([_P, _P, ctypes.c_int, _P], ctypes.c_int),
    "eii_kernel_name": ([ctypes.c_int], ctypes.c_char_p),
    "eii_profile_enable": ([_P, ctypes.c_int], ctypes.c_int),
    "eii_chunk_sequences": ([_P, ctypes.c_int, ctypes.c_int], ctypes.c_int),
    "eii_mma_rate": ([ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                      ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
    "eii_profile_read": ([_P, ctypes.c_int, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)],
                         ctypes.c_int),
    "eii_linear": ([_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P, ctypes.c_int, ctypes.c_int,
                    ctypes.c_int, ctypes.c_int, _P, _P], ctypes.c_int),
    "eii_block_trace": ([_P, ctypes.c_int, _P, ctypes.c_int, _P], ctypes.c_int),
    "eii_set_residual_grid": ([_P, _P, _P], ctypes.c_int),
    "eii_set_residual_grid_channels": ([_P, _P, _P], ctypes.c_int),
    "eii_rmsnorm_trace": ([_P, _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P],
                          ctypes.c_int),
    "eii_table_exp": ([_P], ctypes.c_int),
    "eii_table_silu": ([ctypes.c_int, ctypes.c_int, ctypes.c_int, _P], ctypes.c_int),
    "eii_table_rope": ([ctypes.c_int, _P, _P], ctypes.c_int),
    "eii_verify_tables": ([_P, ctypes.c_size_t], ctypes.c_int),
    "eii_decoder_open": ([_P, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_P)], ctypes.c_int),
    "eii_decoder_prefill": ([_P, _P, ctypes.c_int, _P, _P], ctypes.c_int),
    "eii_decoder_step": ([_P, _P, _P, _P], ctypes.c_int),
    "eii_decoder_step_device": ([_P, _P, _P, ctypes.c_int64, _P, _P], ctypes.c_int),
    "eii_decoder_step_device_async": ([_P, _P, _P, ctypes.c_int64, _P, _P], ctypes.c_int),
    "eii_decoder_sync": ([_P, _P], ctypes.c_int),
    "eii_decoder_position": ([_P], ctypes.c_int),
    "eii_decoder_reset": ([_P], ctypes.c_int),
    "eii_decoder_close": ([_P], None),
    "eii_linear_plan_open": ([_P, _P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.POINTER(_P)], ctypes.c_int),
    "eii_linear_plan_run": ([_P, _P, ctypes.c_int, _P, ctypes.c_int64, _P, _P, _P], ctypes.c_int),
    "eii_linear_plan_close": ([_P], None),
}


# eii_trace (include/eii.h): the sites of Model.block(trace) (python/intref.py:192-286), in struct order
TRACE_SITES = ("resid_in", "norm1_U", "norm1_z", "norm1_out", "q_proj", "k_proj", "v_proj", "q_rope", "k_rope",
               "attn_score", "attn_prob", "attn_ctx", "o_res", "resid_mid", "norm2_U", "norm2_z", "norm2_out",
               "gate_proj", "up_proj", "silu_gate", "mlp_gated", "down_res", "resid_out")


class _Trace(ctypes.Structure):
    _fields_ = [(k, _P) for k in TRACE_SITES]


def trace_shapes(T):
    D, K, F, H = D_MODEL, 192, 1536, 9
    sh = {k: (T, D) for k in TRACE_SITES}
    sh.update(norm1_U=(T,), norm2_U=(T,), k_proj=(T, K), v_proj=(T, K), k_rope=(T, K), attn_score=(H, T, T),
              attn_prob=(H, T, T), gate_proj=(T, F), up_proj=(T, F), silu_gate=(T, F), mlp_gated=(T, F))
    return sh


def lib():
    """Load libeii.so once (raises EiiError if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise EiiError(EII_ERR_CUDA, f"{LIB_PATH} is missing; run __graft_entry__.build() first")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def mma_rate(device, n, noise=0, threads=640, iters=2000):
    """Cycles per tcgen05.mma.kind::i8 (M = 128, N = n, K = 32) with background work `noise` on the
    other warps (include/eii.h, eii_mma_rate)."""
    c = ctypes.c_double()
    check(lib().eii_mma_rate(device, n, noise, threads, iters, ctypes.byref(c)))
    return c.value


def check(rc):
    if rc != EII_OK:
        raise EiiError(rc, lib().eii_last_error().decode(errors="replace"))


def ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


class Engine:
    """One engine handle on one CUDA device (owns the device weights and workspaces)."""

    def __init__(self, model_bin, device=0):
        h = ctypes.c_void_p()
        if isinstance(model_bin, (bytes, bytearray, memoryview, np.ndarray)):
            buf = np.frombuffer(model_bin, dtype=np.uint8) if not isinstance(model_bin, np.ndarray) else model_bin
            check(lib().eii_open_memory(ptr(buf), buf.nbytes, device, ctypes.byref(h)))
        else:
            check(lib().eii_open(os.fsencode(model_bin), device, ctypes.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            lib().eii_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, ids, embed=False, resid=False, logits=True, digests=False):
        """ids [n_seq, T] -> dict of int32 states (exported layouts) and uint64 digests."""
        ids = _c(ids, np.int64)
        if ids.ndim == 1:
            ids = ids[None, :]
        n, T = ids.shape
        out = {}
        e = np.empty((n, T, D_MODEL), np.int32) if embed else None
        r = np.empty((n, N_LAYERS, T, D_MODEL), np.int32) if resid else None
        lg = np.empty((n, T, VOCAB), np.int32) if logits else None
        dg = np.empty(n, np.uint64) if digests else None
        check(lib().eii_forward(self.h, ptr(ids), n, T, ptr(e), ptr(r), ptr(lg), ptr(dg)))
        for k, v in (("embed", e), ("resid", r), ("logits", lg), ("digests", dg)):
            if v is not None:
                out[k] = v
        return out

    def forward_device(self, ids_ptr, n_seq, T, logits_ptr=None, ld=VOCAB, digests_ptr=None, stream=None):
        check(lib().eii_forward_device(self.h, ctypes.c_void_p(ids_ptr), n_seq, T,
                                       ctypes.c_void_p(logits_ptr) if logits_ptr else None, ld,
                                       ctypes.c_void_p(digests_ptr) if digests_ptr else None,
                                       ctypes.c_void_p(stream) if stream else None))

    def chunk_sequences(self, n_seq, T):
        """Sequences per chunk of the engine's workspace for a forward of n_seq x T tokens."""
        cs = lib().eii_chunk_sequences(self.h, n_seq, T)
        if cs < 0:
            check(-cs)
        return cs

    def profile_enable(self, on=True):
        check(lib().eii_profile_enable(self.h, 1 if on else 0))

    def profile_read(self):
        """{kernel name: (total ms, launches)} since the last profile_enable."""
        out = {}
        for k in range(NUM_KERNEL_KINDS):
            ms, n = ctypes.c_double(), ctypes.c_int64()
            check(lib().eii_profile_read(self.h, k, ctypes.byref(ms), ctypes.byref(n)))
            out[lib().eii_kernel_name(k).decode()] = (ms.value, n.value)
        return out

    def embed(self, ids):
        ids = _c(ids, np.int64).reshape(-1)
        x = np.empty((ids.size, D_MODEL), np.int64)
        check(lib().eii_embed(self.h, ptr(ids), ids.size, ptr(x)))
        return x

    def block(self, layer, x, T=None):
        x = _c(x, np.int64)
        rows = x.shape[0]
        T = rows if T is None else T
        out = np.empty_like(x)
        check(lib().eii_block(self.h, layer, ptr(x), rows // T, T, ptr(out)))
        return out

    def set_residual_grid(self, shift_in, shift_out):
        """Narrow residual grid shifts, per layer [30] (k of resid_in|l, resid_out|l) or per layer and
        channel [30, 576]; None, None turns the grid off."""
        if shift_in is None and shift_out is None:
            check(lib().eii_set_residual_grid(self.h, None, None))
            return
        a = _c(shift_in, np.int32)
        b = _c(shift_out, np.int32)
        if a.shape != b.shape or a.shape not in ((N_LAYERS,), (N_LAYERS, D_MODEL)):
            raise EiiError(EII_ERR_ARG, f"grid shifts must be [30] or [30, 576], got {a.shape} and {b.shape}")
        fn = lib().eii_set_residual_grid if a.ndim == 1 else lib().eii_set_residual_grid_channels
        check(fn(self.h, ptr(a), ptr(b)))

    def block_trace(self, layer, x):
        """Model.block(l, x, trace) of one sequence x [T, 576] -> (new residual, {site: int64 array})."""
        x = _c(x, np.int64)
        T = x.shape[0]
        out = {k: np.empty(s, np.int64) for k, s in trace_shapes(T).items()}
        tr = _Trace(*[ctypes.c_void_p(out[k].ctypes.data) for k in TRACE_SITES])
        check(lib().eii_block_trace(self.h, int(layer), ptr(x), T, ctypes.byref(tr)))
        return out["resid_out"].copy(), out

    def rmsnorm(self, x, gain_q, gain_f, f_out, bits_out, want_trace=False):
        """Model.rmsnorm on the GPU; with want_trace, (out, U [rows], z [rows, 576])."""
        x = _c(x, np.int64)
        g = _c(gain_q, np.int64)
        out = np.empty_like(x)
        U = np.empty(x.shape[0], np.int64) if want_trace else None
        z = np.empty_like(x) if want_trace else None
        check(lib().eii_rmsnorm_trace(self.h, ptr(x), x.shape[0], ptr(g), int(gain_f), int(f_out), int(bits_out),
                                      ptr(out), ptr(U), ptr(z)))
        return (out, U, z) if want_trace else out

    def logits(self, x):
        x = _c(x, np.int64)
        out = np.empty((x.shape[0], VOCAB), np.int64)
        check(lib().eii_logits(self.h, ptr(x), x.shape[0], ptr(out)))
        return out

    def linear(self, a, bits_in, W, m, n, f_in, f_out, bits_out, want_acc=True):
        a = _c(a, np.int64)
        W = _c(W, np.int8)
        m = _c(m, np.int64)
        n = _c(n, np.int64)
        M, K = a.shape
        N = W.shape[0]
        out = np.empty((M, N), np.int64)
        acc = np.empty((M, N), np.int64) if want_acc else None
        check(lib().eii_linear(self.h, ptr(a), M, K, int(bits_in), ptr(W), ptr(m), ptr(n), N, int(f_in), int(f_out),
                               int(bits_out), ptr(out), ptr(acc)))
        return out, acc


def table_exp():
    """exp table (python/intref.py:73-78), regenerated independently of mpmath (include/eii.h)."""
    out = np.empty(1537, np.int64)
    check(lib().eii_table_exp(ptr(out)))
    return out


def table_silu(f_in, f_out, bits):
    """SiLU table over the 65536 INT16 inputs (python/intref.py:81-94), regenerated independently."""
    out = np.empty(65536, np.int64)
    check(lib().eii_table_silu(int(f_in), int(f_out), int(bits), ptr(out)))
    return out


def table_rope(n_pos=512):
    """RoPE tables (python/intref.py:97-108) [n_pos, 32] cos and sin, regenerated independently."""
    c = np.empty((n_pos, 32), np.int64)
    s = np.empty((n_pos, 32), np.int64)
    check(lib().eii_table_rope(int(n_pos), ptr(c), ptr(s)))
    return c, s


def verify_tables(model_bin):
    """Regenerate every table of a model.bin (path or bytes) and compare; raises EiiError on a difference."""
    if not isinstance(model_bin, (bytes, bytearray, memoryview, np.ndarray)):
        with open(model_bin, "rb") as f:
            model_bin = f.read()
    buf = np.frombuffer(model_bin, dtype=np.uint8) if not isinstance(model_bin, np.ndarray) else model_bin
    check(lib().eii_verify_tables(ptr(buf), buf.nbytes))


class LinearPlan:
    """Device-resident Model.linear with bound weights (include/eii.h, eii_linear_plan_*):
    out = SAT_bits_out(RS(a W^T m, n + f_in - f_out)) as int32 on device buffers, with optional
    per-row digests of out and of the exact int64 accumulators."""

    def __init__(self, engine, W, m, n, bits_in, f_in, f_out, bits_out):
        W = _c(W, np.int8)
        m = _c(m, np.int64)
        n = _c(n, np.int64)
        N, K = W.shape
        h = ctypes.c_void_p()
        check(lib().eii_linear_plan_open(engine.h, ptr(W), ptr(m), ptr(n), N, K, int(bits_in), int(f_in), int(f_out),
                                         int(bits_out), ctypes.byref(h)))
        self.h = h
        self.engine = engine  # the engine must outlive the plan
        self.N, self.K = N, K

    def run(self, a_ptr, M, out_ptr, ld=None, dig_out_ptr=None, dig_acc_ptr=None, stream=None):
        v = lambda p: ctypes.c_void_p(p) if p else None
        check(lib().eii_linear_plan_run(self.h, ctypes.c_void_p(a_ptr), int(M), ctypes.c_void_p(out_ptr),
                                        int(ld or self.N), v(dig_out_ptr), v(dig_acc_ptr), v(stream)))

    def close(self):
        if self.h:
            lib().eii_linear_plan_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Decoder:
    """Incremental decoding with a K/V cache (include/eii.h, eii_decoder_*), bit-exact with
    recomputation: step t returns row t of Engine.forward on the first t + 1 tokens."""

    def __init__(self, engine, n_seq, max_T):
        h = ctypes.c_void_p()
        check(lib().eii_decoder_open(engine.h, int(n_seq), int(max_T), ctypes.byref(h)))
        self.h = h
        self.engine = engine  # the engine must outlive the decoder
        self.n_seq = int(n_seq)

    def close(self):
        if self.h:
            lib().eii_decoder_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def position(self):
        return lib().eii_decoder_position(self.h)

    def reset(self):
        check(lib().eii_decoder_reset(self.h))

    def prefill(self, ids, logits=True, digests=False):
        """ids [n_seq, T0] -> {"logits": [n_seq, T0, V] int32, "digests": [n_seq] uint64}."""
        ids = _c(ids, np.int64)
        n, T0 = ids.shape
        lg = np.empty((n, T0, VOCAB), np.int32) if logits else None
        dg = np.empty(n, np.uint64) if digests else None
        check(lib().eii_decoder_prefill(self.h, ptr(ids), T0, ptr(lg), ptr(dg)))
        return {k: v for k, v in (("logits", lg), ("digests", dg)) if v is not None}

    def step(self, ids, logits=True, digests=False):
        """ids [n_seq] (one token per sequence) -> {"logits": [n_seq, V] int32, "digests": [n_seq]}."""
        ids = _c(ids, np.int64).reshape(-1)
        lg = np.empty((self.n_seq, VOCAB), np.int32) if logits else None
        dg = np.empty(self.n_seq, np.uint64) if digests else None
        check(lib().eii_decoder_step(self.h, ptr(ids), ptr(lg), ptr(dg)))
        return {k: v for k, v in (("logits", lg), ("digests", dg)) if v is not None}

    def step_device(self, ids_ptr, logits_ptr=None, ld=VOCAB, digests_ptr=None, stream=None):
        check(lib().eii_decoder_step_device(self.h, ctypes.c_void_p(ids_ptr),
                                            ctypes.c_void_p(logits_ptr) if logits_ptr else None, ld,
                                            ctypes.c_void_p(digests_ptr) if digests_ptr else None,
                                            ctypes.c_void_p(stream) if stream else None))

    def step_device_async(self, ids_ptr, logits_ptr=None, ld=VOCAB, digests_ptr=None, stream=None):
        """step_device without waiting: device-side errors surface at the next sync()."""
        check(lib().eii_decoder_step_device_async(self.h, ctypes.c_void_p(ids_ptr),
                                                  ctypes.c_void_p(logits_ptr) if logits_ptr else None, ld,
                                                  ctypes.c_void_p(digests_ptr) if digests_ptr else None,
                                                  ctypes.c_void_p(stream) if stream else None))

    def sync(self, stream=None):
        check(lib().eii_decoder_sync(self.h, ctypes.c_void_p(stream) if stream else None))


def _mix64(z):
    M = np.uint64(0xFFFFFFFFFFFFFFFF)
    with np.errstate(over="ignore"):
        z = (z + np.uint64(0x9E3779B97F4A7C15)) & M
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return (z ^ (z >> np.uint64(31))) | np.uint64(1)


def digest_logits(logits):
    """Host restatement of the device digest (include/eii.h, eii_forward `digests`):
    sum over (t, v) of uint32(logit) * mix64(t) * mix64(2^32 + v), mod 2^64, per sequence."""
    lg = np.asarray(logits)
    n, T, V = lg.shape
    wa = _mix64(np.arange(T, dtype=np.uint64))
    wb = _mix64(np.arange(V, dtype=np.uint64) + np.uint64(1 << 32))
    out = np.empty(n, np.uint64)
    with np.errstate(over="ignore"):
        for s in range(n):
            rows = (lg[s].astype(np.uint32).astype(np.uint64) * wb[None, :]).sum(axis=1, dtype=np.uint64)
            out[s] = (rows * wa).sum(dtype=np.uint64)
    return out
