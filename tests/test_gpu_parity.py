"""Bit-exact parity of the sm_100a engine (through the C ABI) with the reference.

Compared against the committed digests of the reference's own exports (tests/golden) and,
for finer-grained checks and random cases, against the pinned CPU oracle (oracle/)."""
import numpy as np
import pytest

from conftest import golden, sha256_arr
from oracle import forward as ofw
from oracle import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(base_model_path):
    import _eii
    e = _eii.Engine(base_model_path, 0)
    yield e
    e.close()


@pytest.fixture(scope="module")
def eng_outlier(outlier_model_path):
    import _eii
    e = _eii.Engine(outlier_model_path, 0)
    yield e
    e.close()


def oracle_linear(a, bits_in, W, m, n, f_in, f_out, bits_out):
    acc = ofw.matmul_exact(a, W, 1 << (bits_in - 1))
    return ofw.sat(ofw.rs(acc * m[None, :], n + f_in - f_out), bits_out), acc


def first_diff(got, want):
    d = np.argwhere(np.asarray(got) != np.asarray(want))
    return None if d.size == 0 else (tuple(d[0]), int(np.asarray(got)[tuple(d[0])]), int(np.asarray(want)[tuple(d[0])]),
                                     len(d))


# ------------------------------------------------------------------------------ contraction
def test_linear_single_tile(eng, base_model):
    """One 128 x 128 output tile, K = 576, INT16 activations over the full range."""
    q, m, n = base_model["layers"][0]["q"]
    rng = np.random.default_rng(5)
    a = rng.integers(-32768, 32768, size=(128, 576), dtype=np.int64)
    out, acc = eng.linear(a, 16, q[:128], m[:128], n[:128], 13, 10, 16)
    want_out, want_acc = oracle_linear(a, 16, q[:128], m[:128], n[:128], 13, 10, 16)
    assert first_diff(acc, want_acc) is None, first_diff(acc, want_acc)
    assert first_diff(out, want_out) is None


def test_linear_sweep_golden(eng, base_model):
    """Config-5 shapes against the reference's Model.linear digests (tests/golden/gemm_sweep.json)."""
    from test_oracle_golden import sweep_activations
    for c in golden("gemm_sweep.json")["cases"]:
        wname, wl = c["weight"]
        W = (base_model["emb_q"], base_model["emb_m"], base_model["emb_n"]) if wname == "embed" \
            else base_model["layers"][wl][wname]
        a = sweep_activations(c)
        out, acc = eng.linear(a, c["bits_in"], W[0], W[1], W[2], c["f_in"], c["f_out"], c["bits_out"])
        assert sha256_arr(acc, np.int64) == c["acc_sha256"], c["name"]
        assert sha256_arr(out, np.int64) == c["out_sha256"], c["name"]


@pytest.mark.parametrize("M,K,N,bits", [(1, 576, 64, 16), (7, 1536, 192, 32), (129, 576, 576, 16),
                                        (300, 1536, 576, 32), (256, 32, 16, 16), (640, 160, 960, 32)])
def test_linear_ragged_extremes(eng, M, K, N, bits):
    """Ragged M/N/K, extreme activations (all -2^(b-1), all 2^(b-1)-1) and weights (+-127, -128)."""
    rng = np.random.default_rng(M * 7 + K + N + bits)
    lo, hi = -(1 << (bits - 1)), (1 << (bits - 1))
    a = rng.integers(lo, hi, size=(M, K), dtype=np.int64)
    a[0] = lo
    if M > 1:
        a[1] = hi - 1
    W = rng.integers(-128, 128, size=(N, K), dtype=np.int64).astype(np.int8)
    W[0] = -128
    if N > 1:
        W[1] = 127
    m = rng.integers(1 << 13, (1 << 14) + 1, size=N, dtype=np.int64)
    n = rng.integers(18, 30, size=N, dtype=np.int64)
    for bits_out in (16, 32, 64):
        out, acc = eng.linear(a, bits, W, m, n, 12, 10, bits_out)
        want_out, want_acc = oracle_linear(a, bits, W, m, n, 12, 10, bits_out)
        assert first_diff(acc, want_acc) is None, first_diff(acc, want_acc)
        assert first_diff(out, want_out) is None, (bits_out, first_diff(out, want_out))


# ------------------------------------------------------------------------------ steps
def test_embed_and_rmsnorm(eng, base_model):
    ids = synth.window_ids(64, 24)
    x = eng.embed(ids)
    want = ofw.embed(base_model, ids)
    assert first_diff(x, want) is None
    L0 = base_model["layers"][0]
    F = ofw.fm_unpack(L0["fm"])
    rng = np.random.default_rng(9)
    xr = rng.integers(-(1 << 31), 1 << 31, size=(37, 576), dtype=np.int64)
    xr[0] = 0                      # all-zero row: S = 0, only epsilon
    xr[1] = -(1 << 31)             # saturated row
    for x_in in (x, xr):
        got = eng.rmsnorm(x_in, L0["ln1_q"], L0["ln1_f"], F["h"][1], 16)
        exp = ofw.rmsnorm(x_in, L0["ln1_q"], L0["ln1_f"], F["h"][1], 16)
        assert first_diff(got, exp) is None, first_diff(got, exp)


@pytest.mark.parametrize("layer", [0, 4, 11, 13, 28])
def test_block_matches_oracle(eng, base_model, layer):
    """One decoder block (python/intref.py:192-286) on two sequences; layers chosen for their
    formats: INT32 attn_ctx (0, 4), INT32 silu_gate (11, 28), INT16 mlp_gated (13)."""
    T = 24
    ids = np.stack([synth.window_ids(64, T), synth.window_ids(65, T)])
    x = ofw.embed(base_model, ids)
    for l in range(layer):
        x = ofw.block_batch(base_model, l, x, T)
    want = ofw.block_batch(base_model, layer, x, T)
    got = eng.block(layer, x, T)
    assert first_diff(got, want) is None, first_diff(got, want)


# ------------------------------------------------------------------------------ full forward
def _check_set(e, mdl, name):
    g = golden(f"vectors_{name}.json")
    ids = synth.window_ids(g["window"], g["tokens"])
    out = e.forward(ids, embed=True, resid=True, logits=True, digests=True)
    files = g["files"]
    ok_embed = sha256_arr(out["embed"][0], np.int32) == files["exp_embed.i32"]["sha256"]
    ok_resid = sha256_arr(out["resid"][0], np.int32) == files["exp_resid_out.i32"]["sha256"]
    ok_logits = sha256_arr(out["logits"][0], np.int32) == files["exp_logits.i32"]["sha256"]
    if not (ok_embed and ok_resid and ok_logits):
        ref = ofw.forward(mdl, ids)
        msg = [f"embed: {first_diff(out['embed'][0], ref['embed'][0])}"]
        for l in range(30):
            d = first_diff(out["resid"][0, l], ref["resid"][l, 0])
            if d is not None:
                msg.append(f"layer {l}: {d}")
                break
        msg.append(f"logits: {first_diff(out['logits'][0], ref['logits'][0].astype(np.int32))}")
        pytest.fail("; ".join(msg))
    import _eii
    assert out["digests"][0] == _eii.digest_logits(out["logits"])[0]


def test_forward_t24(eng, base_model):
    _check_set(eng, base_model, "t24")


def test_forward_t128(eng, base_model):
    _check_set(eng, base_model, "t128")


def test_forward_t160_outlier(eng_outlier, outlier_model):
    _check_set(eng_outlier, outlier_model, "t160")


def test_batch_subset_against_reference(eng):
    """Config 4 in miniature: golden subset sequences embedded in a larger batch of the same
    4096 x 128 table (other rows in between) must reproduce the reference's per-sequence logits."""
    g = golden("config4_subset.json")
    table = synth.token_table()
    seqs = g["sequences"][:16]
    rows = sorted(set([s["row"] for s in seqs] + list(range(40))))
    ids = table[rows, :g["T"]]
    out = eng.forward(ids, logits=True, digests=True)
    import _eii
    dig = _eii.digest_logits(out["logits"])
    assert np.array_equal(dig, out["digests"])
    for s in seqs:
        i = rows.index(s["row"])
        assert sha256_arr(out["logits"][i], np.int32) == s["logits_i32_sha256"], s["row"]
        assert int(out["logits"][i, -1].argmax()) == s["argmax_last"]


def test_errors_are_reported(eng):
    import _eii
    with pytest.raises(_eii.EiiError) as ei:
        eng.forward(np.array([[0, 49152]], np.int64))
    assert ei.value.code == _eii.EII_ERR_ARG
    with pytest.raises(_eii.EiiError) as ei:
        eng.forward(np.zeros((1, 513), np.int64))
    assert ei.value.code == _eii.EII_ERR_ARG
    # the handle stays usable after a rejected call
    out = eng.forward(synth.window_ids(64, 3), logits=True)
    assert out["logits"].shape == (1, 3, 49152)


@pytest.mark.parametrize("switch", ["EII_O_FEATURE_MAJOR", "EII_DOWN_ROW_MAJOR", "EII_LOGITS_FEATURE_MAJOR", "EII_NO_ACC32",
                                    "EII_NO_NORM_FUSION"])
def test_forward_alternative_gemm_layouts(base_model, base_model_path, outlier_model, outlier_model_path, monkeypatch,
                                          switch):
    """The O projection on the feature-major GEMM (offset-binary context planes from every attention
    kernel), the down projection on the row-major GEMM (signed-digit gated planes), and the tied logits
    on the feature-major GEMM (offset-binary final-norm planes, per-sequence digests): the reference's
    digests for t24 and t160 (the long tensor-core attention), a decode that reaches the decode attention
    kernel, and the per-site trace (the trace's row-major GEMMs read the same planes).  EII_NO_NORM_FUSION:
    the first layer's RMSNorm as its own kernel (by default the embedding kernel produces its planes)."""
    import _eii
    import intref as drop
    from test_oracle_golden import check_trace, trace_inputs
    monkeypatch.setenv(switch, "1")
    e = _eii.Engine(base_model_path, 0)
    try:
        _check_set(e, base_model, "t24")
        _decode_check(e, synth.window_ids(64, 12)[None, :], 6)
    finally:
        e.close()
    e = _eii.Engine(outlier_model_path, 0)
    try:
        _check_set(e, outlier_model, "t160")
    finally:
        e.close()
    g, xs = trace_inputs(base_model)
    M = drop.Model(model_bin=base_model_path)
    for l, x in xs.items():
        tr = {}
        M.block(l, x, trace=tr)
        check_trace(tr, g["layers"][str(l)])


def test_forward_t128_cuda_core_attention(base_model, base_model_path, monkeypatch):
    """The CUDA-core attention kernel (the trace's kernel, and a test switch) is exact too."""
    import _eii
    monkeypatch.setenv("EII_ATTENTION", "cuda_core")
    e = _eii.Engine(base_model_path, 0)
    try:
        _check_set(e, base_model, "t128")
    finally:
        e.close()


# ------------------------------------------------------------------ attention for 128 < T <= 512
def _forward_vs_oracle(e, mdl, ids):
    out = e.forward(ids, resid=True, logits=True)
    for s in range(ids.shape[0]):
        ref = ofw.forward(mdl, ids[s])
        for l in range(30):
            d = first_diff(out["resid"][s, l], ref["resid"][l, 0])
            assert d is None, (s, l, d)
        d = first_diff(out["logits"][s], ref["logits"][0].astype(np.int32))
        assert d is None, (s, d)


def test_forward_t512_matches_oracle(eng, base_model):
    """The longest sequence the reference allows (its RoPE table has 512 rows): four 128-row query
    tiles against up to four key tiles on the tensor cores, every residual and logit exact."""
    _forward_vs_oracle(eng, base_model, synth.window_ids(7, 512)[None, :])


def test_forward_t200_outlier_matches_oracle(eng_outlier, outlier_model):
    """A ragged T (a 72-row last query tile) on the outlier-gain model (saturating scores)."""
    _forward_vs_oracle(eng_outlier, outlier_model, synth.window_ids(100, 200)[None, :])


@pytest.mark.parametrize("T", [129, 257, 300, 384, 511])
def test_long_attention_tensor_core_equals_cuda_core(base_model_path, T):
    """The tensor-core kernel for T > 128 against the CUDA-core kernel on several sequences of the
    same batch (each item a (sequence, head, query tile)), logits and per-sequence digests."""
    import _eii
    table = synth.token_table()
    ids = table[3:8, :T]
    e = _eii.Engine(base_model_path, 0)
    try:
        tc = e.forward(ids, logits=True, digests=True)
    finally:
        e.close()
    import os
    old = os.environ.get("EII_ATTENTION")
    os.environ["EII_ATTENTION"] = "cuda_core"
    try:
        e = _eii.Engine(base_model_path, 0)
        try:
            cc = e.forward(ids, logits=True, digests=True)
        finally:
            e.close()
    finally:
        if old is None:
            del os.environ["EII_ATTENTION"]
        else:
            os.environ["EII_ATTENTION"] = old
    assert np.array_equal(tc["digests"], cc["digests"])
    assert first_diff(tc["logits"], cc["logits"]) is None


def test_decode_long_prompt_base_model(eng):
    """Prompt of 260 tokens (three query tiles in the prefill), then 40 decoding steps."""
    _decode_check(eng, np.stack([synth.window_ids(11, 300), synth.window_ids(12, 300)]), 260)


@pytest.mark.parametrize("layer", [0, 11])
def test_block_full_silu_table(base_model, base_model_path, monkeypatch, layer):
    """The gate/up epilogue's fallback that gathers from the full 65536-entry SiLU table (used when
    the compact shared-memory form does not apply) is exact too."""
    import _eii
    monkeypatch.setenv("EII_SILU", "global")
    e = _eii.Engine(base_model_path, 0)
    try:
        T = 24
        x = ofw.embed(base_model, synth.window_ids(64, T))
        for l in range(layer):
            x = ofw.block_batch(base_model, l, x, T)
        want = ofw.block_batch(base_model, layer, x, T)
        got = e.block(layer, x, T)
        assert first_diff(got, want) is None, first_diff(got, want)
    finally:
        e.close()


def test_forward_t24_generic_requant(base_model, base_model_path, monkeypatch):
    """The int64 epilogue path (taken when a column shift is outside [1, 31] or a multiplier is
    >= 2^15) gives the same integers as the fast 32-bit path."""
    import _eii
    monkeypatch.setenv("EII_GENERIC_REQUANT", "1")
    e = _eii.Engine(base_model_path, 0)
    try:
        _check_set(e, base_model, "t24")
    finally:
        e.close()


def test_forward_t128_generic_attention_requant(base_model, base_model_path, monkeypatch):
    """The tensor-core attention's 64-bit score and context requantisation (taken for shifts outside
    [8, 31]) and its 32-bit forms give the same integers."""
    import _eii
    monkeypatch.setenv("EII_ATTENTION", "generic")
    e = _eii.Engine(base_model_path, 0)
    try:
        _check_set(e, base_model, "t128")
    finally:
        e.close()


def test_forward_t24_generic_norm(base_model, base_model_path, monkeypatch):
    """The generic RMSNorm kernel (int64 outputs, any plane count and shift) and the lean two-plane
    kernel the forward pass uses give the same integers."""
    import _eii
    monkeypatch.setenv("EII_NORM", "generic")
    e = _eii.Engine(base_model_path, 0)
    try:
        _check_set(e, base_model, "t24")
    finally:
        e.close()


def test_forward_t24_without_narrow_requant(base_model, base_model_path, monkeypatch):
    """The 32-bit requantisation with explicit 64-bit saturation tests (used when a column's bound
    does not prove that the shifted value fits int32) gives the same integers."""
    import _eii
    monkeypatch.setenv("EII_NO_NARROW", "1")
    e = _eii.Engine(base_model_path, 0)
    try:
        _check_set(e, base_model, "t24")
    finally:
        e.close()


def test_forward_t128_without_programmatic_launch(base_model, base_model_path, monkeypatch):
    """Kernels launched plainly (EII_PDL=0) and with programmatic stream serialization give the
    same integers (each kernel waits for its predecessor before touching its outputs)."""
    import _eii
    monkeypatch.setenv("EII_PDL", "0")
    e = _eii.Engine(base_model_path, 0)
    try:
        _check_set(e, base_model, "t128")
    finally:
        e.close()


# ------------------------------------------------------------------------------ incremental decoding
def _decode_check(eng, ids, T0):
    """Prefill T0 tokens, decode the rest one token per step; every logits row must equal the full
    forward's, and the prefill and step digests must add up to the forward digest."""
    import _eii
    n, T = ids.shape
    ref = eng.forward(ids, logits=True, digests=True)
    dec = _eii.Decoder(eng, n, T)
    try:
        total = np.zeros(n, np.uint64)
        if T0 > 0:
            out = dec.prefill(ids[:, :T0], logits=True, digests=True)
            assert np.array_equal(out["logits"], ref["logits"][:, :T0])
            total += out["digests"]
        assert dec.position == T0
        for t in range(T0, T):
            out = dec.step(ids[:, t], logits=True, digests=True)
            d = first_diff(out["logits"], ref["logits"][:, t])
            assert d is None, (t, d)
            total += out["digests"]
        assert dec.position == T
        assert np.array_equal(total, ref["digests"])
        with pytest.raises(_eii.EiiError) as ei:
            dec.step(ids[:, 0])
        assert ei.value.code == _eii.EII_ERR_ARG  # the cache is full
    finally:
        dec.close()


def test_decode_matches_recomputation(eng):
    ids = np.stack([synth.window_ids(64, 24), synth.window_ids(65, 24), synth.window_ids(66, 24)])
    _decode_check(eng, ids, 5)


def test_decode_from_empty_cache(eng):
    _decode_check(eng, synth.window_ids(70, 9)[None, :], 0)


def test_decode_across_staged_limit(eng):
    """Steps at L = 121 .. 128 keys run the staged decode kernel, L = 129 .. 136 the general one; both
    append their step's K/V row to the cache that the other then reads."""
    _decode_check(eng, np.stack([synth.window_ids(80, 136), synth.window_ids(81, 136)]), 120)


def test_decode_unstaged_kernel(base_model_path, monkeypatch):
    """EII_DECODE_UNSTAGED: the general decode kernel at L <= 128, where steps otherwise take the
    staged one, from an empty cache and after a prompt."""
    import _eii
    monkeypatch.setenv("EII_DECODE_UNSTAGED", "1")
    e = _eii.Engine(base_model_path, 0)
    try:
        _decode_check(e, synth.window_ids(70, 9)[None, :], 0)
        _decode_check(e, np.stack([synth.window_ids(64, 40), synth.window_ids(65, 40)]), 30)
    finally:
        e.close()


def test_decode_async_steps_and_deferred_errors(eng, base_model):
    """eii_decoder_step_device_async: steps enqueued back to back on a side stream give the forward's
    logits rows and digests after eii_decoder_sync; a token id outside the vocabulary in an enqueued
    step is reported by the next sync (EII_ERR_ARG), and the engine works again afterwards."""
    import torch
    import _eii
    ids = np.stack([synth.window_ids(70 + i, 16) for i in range(3)])
    n, T = ids.shape
    T0 = 9
    ref = eng.forward(ids, logits=True, digests=True)
    dec = _eii.Decoder(eng, n, T)
    try:
        pre = dec.prefill(ids[:, :T0], logits=False, digests=True)["digests"]
        side = torch.cuda.Stream()
        ids_d = torch.from_numpy(np.ascontiguousarray(ids[:, T0:].T)).cuda()
        lg = torch.empty((T - T0, n, _eii.VOCAB), dtype=torch.int32, device="cuda")
        dg = torch.zeros((T - T0, n), dtype=torch.int64, device="cuda")
        with torch.cuda.stream(side):
            for t in range(T - T0):
                dec.step_device_async(ids_d[t].data_ptr(), lg[t].data_ptr(), _eii.VOCAB, dg[t].data_ptr(), side.cuda_stream)
        dec.sync(side.cuda_stream)
        assert dec.position == T
        for t in range(T - T0):
            d = first_diff(lg[t].cpu().numpy(), ref["logits"][:, T0 + t])
            assert d is None, (t, d)
        total = pre.view(np.uint64) + dg.sum(dim=0).cpu().numpy().view(np.uint64)
        assert np.array_equal(total, ref["digests"])
        dec.reset()
        dec.prefill(ids[:, :T0], logits=False)
        bad = torch.tensor([0, _eii.VOCAB, 1], dtype=torch.int64, device="cuda")
        with torch.cuda.stream(side):
            dec.step_device_async(bad.data_ptr(), lg[0].data_ptr(), _eii.VOCAB, None, side.cuda_stream)
        with pytest.raises(_eii.EiiError) as ei:
            dec.sync(side.cuda_stream)
        assert ei.value.code == _eii.EII_ERR_ARG
    finally:
        dec.close()
    _check_set(eng, base_model, "t24")


def test_decode_outlier_model_long_prompt(eng_outlier):
    """T = 160 (the long tensor-core attention kernel for the prompt): prompt 150, then 10 steps."""
    g = golden("vectors_t160.json")
    ids = synth.window_ids(g["window"], g["tokens"])[None, :]
    _decode_check(eng_outlier, ids, 150)


def test_decoder_arguments(eng):
    import _eii
    with pytest.raises(_eii.EiiError):
        _eii.Decoder(eng, 2, 513)
    dec = _eii.Decoder(eng, 2, 8)
    try:
        with pytest.raises(_eii.EiiError):
            dec.prefill(np.zeros((2, 9), np.int64))
        dec.prefill(np.zeros((2, 3), np.int64), logits=False)
        with pytest.raises(_eii.EiiError):
            dec.prefill(np.zeros((2, 3), np.int64), logits=False)  # prefill comes first
        with pytest.raises(_eii.EiiError):
            dec.step(np.array([0, 49152], np.int64))
        dec.reset()
        assert dec.position == 0
    finally:
        dec.close()


# ------------------------------------------------------------------------------ per-site trace
def test_block_trace_matches_reference(base_model, base_model_path):
    """Model.block(l, x, trace) of the drop-in module (eii_block_trace) against the digests of the
    reference's own trace of every site, at five layers (every format variant)."""
    import intref as drop
    from test_oracle_golden import check_trace, trace_inputs
    g, xs = trace_inputs(base_model)
    M = drop.Model(model_bin=base_model_path)
    for l, x in xs.items():
        tr = {}
        out = M.block(l, x, trace=tr)
        check_trace(tr, g["layers"][str(l)])
        assert np.array_equal(out, tr["resid_out"])


# ------------------------------------------------------------------------------ narrow comparison mode
@pytest.mark.parametrize("wide,nres", [(False, False), (False, True), (True, True)])
def test_narrow_modes_match_reference(base_model_path, wide, nres):
    """Model(wide).forward(ids, narrow_residual) of the drop-in module against the reference's own
    logits digests (python/intref.py:152-160, 288-308) on the t24 tokens."""
    import intref as drop
    g = golden("narrow_t24.json")
    want = g["modes"][f"wide={int(wide)},narrow_residual={int(nres)}"]
    M = drop.Model(wide=wide, model_bin=base_model_path)
    try:
        lg = M.forward(synth.window_ids(g["window"], g["tokens"]), narrow_residual=nres)
    finally:
        M.close()
    assert lg[0, :8].tolist() == want["logits_row0_first8"]
    assert sha256_arr(lg, np.int64) == want["logits_int64_sha256"]


def test_forward_t24_unsigned_gated_planes(base_model, base_model_path, monkeypatch):
    """The down GEMM on the plain gated byte planes (EII_NO_SD: no signed digits, all four planes
    every tile) gives the same integers as the signed-digit planes with the top plane skipped."""
    import _eii
    monkeypatch.setenv("EII_NO_SD", "1")
    e = _eii.Engine(base_model_path, 0)
    try:
        _check_set(e, base_model, "t24")
    finally:
        e.close()


def test_chunk_sequences_equal_chunks(eng, monkeypatch):
    """Without EII_CHUNK_ROWS the sequences are split into the fewest chunks of at most 65536 rows,
    all of (nearly) equal size (no small remainder chunk); the variable sets the chunk exactly; the
    count never exceeds the request."""
    import _eii
    monkeypatch.delenv("EII_CHUNK_ROWS", raising=False)
    assert eng.chunk_sequences(4096, 128) == 512   # 8 chunks of 512 (one GPU)
    assert eng.chunk_sequences(512, 128) == 512    # the shard of one of 8 GPUs: one chunk
    assert eng.chunk_sequences(513, 128) == 257    # two chunks of 257 and 256, not 512 + 1
    assert eng.chunk_sequences(3, 128) == 3
    assert eng.chunk_sequences(160, 512) == 80     # 128 sequences fit 65536 rows: two chunks of 80
    for n, T in ((4096, 128), (1000, 160), (100000, 1), (7, 512)):
        cs = eng.chunk_sequences(n, T)
        chunks = -(-n // cs)
        assert cs * T <= 65536 or cs == 1
        assert n - (chunks - 1) * cs >= cs - chunks   # the last chunk is within one sequence per chunk
    monkeypatch.setenv("EII_CHUNK_ROWS", "16384")
    assert eng.chunk_sequences(4096, 128) == 128
    with pytest.raises(_eii.EiiError):
        eng.chunk_sequences(0, 128)


def test_bounded_wait_timeout_reports_error_and_recovers(eng, monkeypatch):
    """The bounded mbarrier waits: with EII_TEST_STALL_NS set, eii_linear's epilogue warps first wait
    on a barrier nothing arrives on; the wait gives up after 2 ms, the CTA aborts (producer and MMA
    thread drain their copies and MMAs before TMEM is freed) and the call reports EII_ERR_DEVICE.
    The same handle then gives bit-exact results."""
    import _eii
    rng = np.random.default_rng(11)
    a = rng.integers(-32768, 32768, size=(300, 576), dtype=np.int64)
    W = rng.integers(-127, 128, size=(192, 576), dtype=np.int64).astype(np.int8)
    m = rng.integers(1 << 13, (1 << 14) + 1, size=192, dtype=np.int64)
    n = rng.integers(18, 30, size=192, dtype=np.int64)
    monkeypatch.setenv("EII_TEST_STALL_NS", "2000000")
    with pytest.raises(_eii.EiiError) as ei:
        eng.linear(a, 16, W, m, n, 12, 10, 16)
    assert ei.value.code == _eii.EII_ERR_DEVICE and "104" in str(ei.value)
    monkeypatch.delenv("EII_TEST_STALL_NS")
    out, acc = eng.linear(a, 16, W, m, n, 12, 10, 16)
    want_out, want_acc = oracle_linear(a, 16, W, m, n, 12, 10, 16)
    assert first_diff(acc, want_acc) is None and first_diff(out, want_out) is None
