"""The contraction sweep (Model.linear, python/intref.py:186-190) at M = 512 ... 262144 rows through
eii_linear_plan_run, against the block digests of the reference's own Model.linear
(tests/golden/gemm_sweep_large.json, written by make_golden.py --only-sweep).

Every row's int32 output and exact int64 accumulator enter a digest on the device; the host folds
the per-row digests into 4096-row block digests, so a mismatch names the block it sits in."""
import numpy as np
import pytest

import sweep
from conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(base_model_path):
    import _eii
    e = _eii.Engine(base_model_path, 0)
    yield e
    e.close()


def _run_case(eng, model_bin, c):
    import torch
    import _eii
    ci, M = c["case"], c["M"]
    W, m, n = sweep.weights(model_bin, ci)
    bits_in, f_in, f_out, bits_out = sweep.case_formats(ci)
    assert (bits_in, f_in, f_out, bits_out) == (c["bits_in"], c["f_in"], c["f_out"], c["bits_out"])
    N, K = W.shape
    a = torch.empty((M, K), dtype=torch.int32, device="cuda")
    for b in range(sweep.blocks(M)):
        blk = sweep.activation_block(ci, M, b, K, bits_in)
        a[sweep.BLOCK * b:sweep.BLOCK * b + blk.shape[0]].copy_(torch.from_numpy(blk))
    out = torch.empty((M, N), dtype=torch.int32, device="cuda")
    dig_out = torch.empty(M, dtype=torch.int64, device="cuda")
    dig_acc = torch.empty(M, dtype=torch.int64, device="cuda")
    plan = _eii.LinearPlan(eng, W, m, n, bits_in, f_in, f_out, bits_out)
    try:
        torch.cuda.synchronize()
        plan.run(a.data_ptr(), M, out.data_ptr(), N, dig_out.data_ptr(), dig_acc.data_ptr())
    finally:
        plan.close()
    first8 = out[2, :8].cpu().numpy().tolist()
    da = sweep.block_digests(dig_acc.cpu().numpy().view(np.uint64), M)
    do = sweep.block_digests(dig_out.cpu().numpy().view(np.uint64), M)
    del a, out
    torch.cuda.empty_cache()
    return first8, sweep.hexes(da), sweep.hexes(do)


def _cases(big):
    return [c for c in golden("gemm_sweep_large.json")["cases"] if (c["M"] == max(sweep.MS)) == big]


@pytest.mark.parametrize("c", _cases(False), ids=lambda c: f"{c['name']}-M{c['M']}")
def test_sweep_matches_reference(eng, base_model_path, c):
    first8, da, do = _run_case(eng, base_model_path, c)
    assert first8 == c["out_row2_first8"]
    bad = [b for b in range(len(da)) if da[b] != c["acc_blocks"][b]]
    assert not bad, f"acc digests differ in blocks {bad[:8]}"
    bad = [b for b in range(len(do)) if do[b] != c["out_blocks"][b]]
    assert not bad, f"out digests differ in blocks {bad[:8]}"


@pytest.mark.parametrize("c", _cases(True), ids=lambda c: f"{c['name']}-M{c['M']}")
def test_sweep_matches_reference_262144_rows(eng, base_model_path, c):
    """The largest size of the sweep: 262144 rows (51.5 GB of int32 outputs for the logits shape)."""
    first8, da, do = _run_case(eng, base_model_path, c)
    assert first8 == c["out_row2_first8"]
    assert da == c["acc_blocks"], "acc digests differ"
    assert do == c["out_blocks"], "out digests differ"


@pytest.mark.parametrize("ci", range(len(sweep.CASES)), ids=[c[0] for c in sweep.CASES])
def test_sweep_without_digests_equals_with(eng, base_model_path, ci):
    """A plan run without digests (the timed launches; at four planes a kernel compiled without the
    digest code) writes the same int32 outputs as the run with digests, which the reference pins."""
    import torch
    import _eii
    M = 4096 + 96  # a ragged last row block
    W, m, n = sweep.weights(base_model_path, ci)
    bits_in, f_in, f_out, bits_out = sweep.case_formats(ci)
    N, K = W.shape
    a = torch.cat([torch.from_numpy(sweep.activation_block(ci, M, b, K, bits_in)) for b in range(sweep.blocks(M))]).cuda()
    out_d = torch.empty((M, N), dtype=torch.int32, device="cuda")
    out_n = torch.full((M, N), -7, dtype=torch.int32, device="cuda")
    dig_out = torch.empty(M, dtype=torch.int64, device="cuda")
    dig_acc = torch.empty(M, dtype=torch.int64, device="cuda")
    plan = _eii.LinearPlan(eng, W, m, n, bits_in, f_in, f_out, bits_out)
    try:
        plan.run(a.data_ptr(), M, out_d.data_ptr(), N, dig_out.data_ptr(), dig_acc.data_ptr())
        plan.run(a.data_ptr(), M, out_n.data_ptr(), N)
        torch.cuda.synchronize()
    finally:
        plan.close()
    assert torch.equal(out_d, out_n)


def test_plan_rejects_out_of_range_activation(eng, base_model_path):
    """A value outside the input format is an argument error (reported by the split kernel), and
    the plan gives exact results afterwards."""
    import torch
    import _eii
    W, m, n = sweep.weights(base_model_path, 0)
    bits_in, f_in, f_out, bits_out = sweep.case_formats(0)
    N, K = W.shape
    a_np = sweep.activation_block(0, 512, 0, K, bits_in)
    a = torch.from_numpy(a_np).cuda()
    out = torch.empty((512, N), dtype=torch.int32, device="cuda")
    plan = _eii.LinearPlan(eng, W, m, n, bits_in, f_in, f_out, bits_out)
    try:
        bad = a.clone()
        bad[7, 3] = 40000
        with pytest.raises(_eii.EiiError) as ei:
            plan.run(bad.data_ptr(), 512, out.data_ptr())
        assert ei.value.code == _eii.EII_ERR_ARG
        plan.run(a.data_ptr(), 512, out.data_ptr())
        from oracle import forward as ofw
        acc = ofw.matmul_exact(a_np.astype(np.int64), W, 1 << (bits_in - 1))
        want = ofw.sat(ofw.rs(acc * m[None, :], n + f_in - f_out), bits_out)
        assert np.array_equal(out.cpu().numpy(), want)
    finally:
        plan.close()


@pytest.mark.parametrize("switch", ["EII_TGEMM_WIDE", "EII_TGEMM_STREAM", "EII_SWEEP_ROW_MAJOR"])
def test_sweep_alternative_paths_match_reference(base_model_path, monkeypatch, switch):
    """The contraction's other code paths against the same reference digests: the feature-major GEMM
    with 64-bit requantisation (EII_TGEMM_WIDE) and with streamed instead of resident activation planes
    (EII_TGEMM_STREAM), and the row-major GEMM (EII_SWEEP_ROW_MAJOR)."""
    import _eii
    monkeypatch.setenv(switch, "1")
    e = _eii.Engine(base_model_path, 0)
    try:
        for c in _cases(False):
            if c["M"] > 4096:
                continue
            first8, da, do = _run_case(e, base_model_path, c)
            assert first8 == c["out_row2_first8"], (switch, c["name"], c["M"])
            assert da == c["acc_blocks"] and do == c["out_blocks"], (switch, c["name"], c["M"])
    finally:
        e.close()
