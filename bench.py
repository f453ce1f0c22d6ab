"""Throughput benchmark of the B200 engine on BASELINE config 4 (the batched-throughput config).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...          (one process per GPU)

Workload: 4096 independent sequences of 128 uniform-random token ids (rows 0..4095 of the seeded
token table) through the integer SmolLM2-135M forward pass of python/intref.py on the seeded
synthetic model, full int32 logits kept in HBM.  Sequences are sharded evenly over the ranks
(total work fixed, so "scaling" is "strong"); ranks exchange nothing on the data path; NCCL only
gathers integer outputs (per-sequence digests and the parity verdict) to rank 0.

One step = one pass of the rank's shard.  `value` is timed with the ids already in HBM and the
logits written to a device buffer; `e2e` repeats the K steps through the C ABI with host
buffers (pinned ids uploaded and per-sequence digests read back inside the timed region).
After timing, the logits of the 64-sequence check subset are compared with the digests the
reference's own intref.py produced (tests/golden/config4_subset.json).

`--impl reference` times the reference's own scalar C program (c/intref.c, built into
oracle/_ref by oracle/build_ref.sh) on the host cores: each step runs one 128-token sequence of
the same workload per host thread, in parallel processes.
"""
import argparse
import datetime
import hashlib
import json
import os
import re
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "exact-integer-inference_b200")
sys.path.insert(0, PKG)

N_SEQ, T, VOCAB, D = 4096, 128, 49152, 576
METRIC = "bit-exact tokens/sec"
UNIT = "tokens/s"
WORKLOAD = "config4: 4096 sequences x 128 tokens, integer SmolLM2-135M forward, full int32 logits"
DATA = "synthetic: seeded N(0,0.02^2) weights through the reference quantiser, uniform token ids"
MODEL_DIR = os.path.join(REPO, "_build", "bench")
REF_BIN = os.path.join(REPO, "oracle", "_ref", "intref")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def rank_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def model_path():
    return os.path.join(MODEL_DIR, "model.bin")


def ensure_model():
    import synthetic
    p = model_path()
    if not os.path.exists(p):
        os.makedirs(MODEL_DIR, exist_ok=True)
        t0 = time.time()
        synthetic.write_model_bin(p)
        log(f"[bench] synthetic model.bin written in {time.time() - t0:.1f} s")
    return p


def token_table():
    import synthetic
    return synthetic.token_table()


def shard(rank, world):
    per = N_SEQ // world
    return rank * per, per


# ------------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception as ex:  # nvidia-smi missing: report no samples
            log(f"[bench] clock sampling unavailable: {ex}")
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.file:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), parts[4:9]))
                except ValueError:
                    continue
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(1, 5) if r[2][i].lower() == "active"})
        sm = sorted(r[0] for r in rows)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": rows[0][1], "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------------ CPU
def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def write_vector_dirs(root, model_bin, seqs):
    """seqs: list of (ids [T], embed [T,576], resid [30,T,576], logits [T,V]) -> vector dirs in the
    layout of python/export_vectors.py, for the reference's C checker."""
    dirs = []
    for i, (ids, emb, res, lg) in enumerate(seqs):
        d = os.path.join(root, f"s{i}")
        os.makedirs(d, exist_ok=True)
        np.asarray(ids, np.int64).tofile(os.path.join(d, "ids.i64"))
        np.asarray(emb, np.int32).tofile(os.path.join(d, "exp_embed.i32"))
        np.asarray(res, np.int32).tofile(os.path.join(d, "exp_resid_out.i32"))
        np.asarray(lg, np.int32).tofile(os.path.join(d, "exp_logits.i32"))
        link = os.path.join(d, "model.bin")
        if not os.path.exists(link):
            os.symlink(model_bin, link)
        dirs.append(d)
    return dirs


def run_reference_c(dirs, procs):
    """Run `procs` reference C processes in parallel (one vector dir each, cycled) and return
    (tokens/s, per-process seconds, verdict lines).  The reference program's own timer covers the
    forward pass and its comparisons, not the model load (c/intref.c:225,256)."""
    t0 = time.time()
    ps = [subprocess.Popen([REF_BIN, dirs[i % len(dirs)]], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
          for i in range(procs)]
    outs = [p.communicate()[0] for p in ps]
    wall = time.time() - t0
    secs, verdicts = [], []
    for o in outs:
        last = o.strip().splitlines()[-1] if o.strip() else ""
        verdicts.append(last)
        m = re.search(r"\((\d+) tokens, ([0-9.]+) s\)", last)
        secs.append(float(m.group(2)) if m else wall)
    return procs * T / max(secs), secs, verdicts, wall


def reference_vectors(model_bin, rows, workdir):
    """Expected states for the reference C program, from the numpy port of intref.py (oracle/)."""
    sys.path.insert(0, REPO)
    from oracle import forward as ofw
    from oracle.modelbin import read_model_bin
    mdl = read_model_bin(model_bin)
    ids = token_table()[rows, :T]
    out = ofw.forward(mdl, ids)
    seqs = [(ids[i], out["embed"][i], out["resid"][:, i], out["logits"][i]) for i in range(len(rows))]
    return write_vector_dirs(workdir, model_bin, seqs)


def cpu_baseline_from_gpu(eng, model_bin, workdir, seconds_hint=30):
    """cpu_baseline leg: the reference C program on a bounded sample (one 128-token sequence per
    host thread), with expected states taken from this engine's own (bit-exact) outputs, so the
    reference program also re-checks them."""
    if not os.path.exists(REF_BIN):
        return None
    procs = min(cpu_threads(), 64)
    rows = list(range(min(4, procs)))
    ids = token_table()[rows, :T]
    out = eng.forward(ids, embed=True, resid=True, logits=True)
    seqs = [(ids[i], out["embed"][i], out["resid"][i], out["logits"][i]) for i in range(len(rows))]
    dirs = write_vector_dirs(workdir, model_bin, seqs)
    tps, secs, verdicts, wall = run_reference_c(dirs, procs)
    exact = sum("ALL STATES EXACT" in v for v in verdicts)
    return {"value": round(tps, 2), "unit": UNIT, "cores": procs, "kind": "reference",
            "sample": f"{procs} sequences x {T} tokens of config 4 (rows {rows[0]}..{rows[-1]} cycled), one per process, "
                      f"c/intref.c -O2 single-threaded each; its own per-process timer (forward + comparisons)",
            "seconds_per_sequence": round(float(np.median(secs)), 2),
            "reference_checked_engine_output": f"{exact}/{procs} ALL STATES EXACT"}


def cpu_baseline_numpy(eng, model_bin, n=24):
    """The numpy path beside the scalar C one: oracle/forward.py (a numpy restatement of
    python/intref.py; the reference's own module is not on the GPU box) timed on the host's cores
    with all BLAS threads, on n sequences of config 4.  Its logits are compared with this engine's."""
    sys.path.insert(0, REPO)
    from oracle import forward as ofw
    from oracle.modelbin import read_model_bin
    mdl = read_model_bin(model_bin)
    ids = token_table()[:n, :T]
    t0 = time.time()
    out = ofw.forward(mdl, ids, want_states=False)
    dt = time.time() - t0
    mine = eng.forward(ids, logits=True)["logits"]
    same = sum(bool(np.array_equal(out["logits"][i], mine[i].astype(np.int64))) for i in range(n))
    return {"value": round(n * T / dt, 2), "unit": UNIT, "cores": cpu_threads(), "kind": "port",
            "sample": f"{n} sequences x {T} tokens of config 4 (rows 0..{n - 1}), one process: oracle/forward.py, "
                      f"numpy with float64 BLAS on all host threads (exact under the bound python/intref.py:61 asserts)",
            "seconds": round(dt, 2), "engine_logits_equal": f"{same}/{n}"}


# ------------------------------------------------------------------------------------ roofline
def roofline(prof, rows_total, peaks, kernel=None):
    """Dominant kernel (most device time in the profiled step), or the named one, against its
    roofline.  The work per launch is the step's total work of that kernel over its launch count
    (chunks may differ in size)."""
    name, (ms, n) = max(prof.items(), key=lambda kv: kv[1][0]) if kernel is None else (kernel, prof[kernel])
    per_launch_s = ms / n / 1e3
    L = 30  # layers: one launch of each layer kernel per layer and chunk; norms 2 per layer + final
    rows = rows_total
    macs_total = {"gemm_gateup_silu": L * rows * 3072 * 576, "gemm_qkv_rope": L * rows * 960 * 576,
                  "gemm_o_resid": L * rows * 576 * 576, "gemm_down_resid": L * rows * 576 * 1536,
                  "gemm_logits": rows * VOCAB * 576,
                  "attention": L * (rows // T) * 9 * 64 * 2 * (T * (T + 1) // 2)}
    bytes_total = {"rmsnorm": (2 * L + 1) * rows * (D * 4 + D * 2), "embed": rows * D * 5}
    macs = {k: v // n for k, v in macs_total.items()}
    bytes_ = {k: v // n for k, v in bytes_total.items()}
    r = rows * (1 if name in ("gemm_logits", "embed") else (2 * L + 1 if name == "rmsnorm" else L)) // n
    int8_peak = 2.0 * peaks.get("bf16_tflops", 1590.0)
    if name in macs:
        achieved = 2.0 * macs[name] / per_launch_s / 1e12
        out = {"kernel": name, "bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1),
               "unit": "TFLOP/s", "frac": round(achieved / int8_peak, 4),
               "peak_note": "int8 dense = 2 x measured bf16 (MEASURED_PEAKS.json), of measured",
               "ops_per_launch": 2 * macs[name], "ops_note": "2 x logical int8-weight x wide-activation MACs"}
    else:
        achieved = bytes_[name] / per_launch_s / 1e9
        out = {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks.get("hbm_gbs", 6650.0),
               "unit": "GB/s", "frac": round(achieved / peaks.get("hbm_gbs", 6650.0), 4), "peak_note": "of measured"}
    out["launch_us"] = round(per_launch_s * 1e6, 1)
    out["rows_per_launch"] = r
    out["traffic"] = traffic_for(name, r)
    act = tensor_active_for(name)
    if act is not None:
        out["tensor_pipe_active_ncu"] = act
    return out


def tensor_active_for(kernel):
    """Tensor-pipe active fraction of the kernel in the committed ncu capture (profiles/traffic.json;
    sm__pipe_tensor_subpipe_imma_cycles_active), byte planes included."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f)[kernel]["tensor_active_pct"] / 100.0
    except Exception:
        return None


def traffic_for(kernel, rows):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.json), scaled by rows."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(p) as f:
            t = json.load(f)
        e = t[kernel]
        return int(e["dram_bytes"] * rows / e["rows"])
    except Exception:
        return None


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


# ------------------------------------------------------------------------------------ arms
def decode_bench(eng, ids_host, ids_dev, ns, fwd_digests, stream, barrier, max_over_ranks):
    """Incremental decoding of this shard: a prompt of T/2 tokens (eii_decoder_prefill), then one token
    per sequence per step (eii_decoder_step_device) to T.  The first step is warm-up; the others are
    timed with CUDA events (max over ranks).  Exactness: the prompt and step digests must add up to
    the digests of the full forward pass timed above (equal logits rows give equal sums)."""
    import torch
    import _eii
    T0 = T // 2
    dec = _eii.Decoder(eng, ns, T)
    try:
        pre = dec.prefill(ids_host[:, :T0], logits=False, digests=True)["digests"]
        ids_t = ids_dev[:, T0:].t().contiguous()  # [T - T0, ns]: the token of each step
        step_logits = torch.empty((ns, VOCAB), dtype=torch.int32, device="cuda")
        step_dig = torch.zeros((T - T0, ns), dtype=torch.int64, device="cuda")
        dec.step_device(ids_t[0].data_ptr(), step_logits.data_ptr(), VOCAB, step_dig[0].data_ptr(), stream)
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for t in range(1, T - T0):  # enqueued back to back; device-side errors surface at sync()
            dec.step_device_async(ids_t[t].data_ptr(), step_logits.data_ptr(), VOCAB, step_dig[t].data_ptr(), stream)
        ev1.record()
        torch.cuda.synchronize()
        dec.sync(stream)
        ms = max_over_ranks(ev0.elapsed_time(ev1))
        total = (torch.from_numpy(pre.view(np.int64).copy()).cuda() + step_dig.sum(dim=0)).cpu().numpy()
        exact = bool(np.array_equal(total, fwd_digests.cpu().numpy()))
    finally:
        dec.close()
    return {"unit": UNIT, "n_seq": N_SEQ, "prompt_tokens": T0, "timed_steps": T - T0 - 1, "ms": round(ms, 3),
            "ms_per_step": round(ms / (T - T0 - 1), 3),
            "path": "eii_decoder_prefill, then eii_decoder_step_device_async (K/V cache, one token per sequence per "
                    "step, steps enqueued back to back) and eii_decoder_sync",
            "exact_vs_forward_digests": exact}


def gemm_sweep_bench(eng, peaks, reps=5):
    """The stand-alone contraction sweep (shapes, formats and activations of
    sweep.py): per (shape, M) the device time of the GEMM kernel (engine profile events on its stream,
    L2 flushed between launches), logical int8-weight x wide-activation ops per second against the
    int8 dense peak, the plane-expanded tensor work (planes x logical ops) against the same peak, and
    exactness: block digests of out and of the exact acc against the reference's own Model.linear
    (tests/golden/gemm_sweep_large.json)."""
    import torch
    import _eii
    import sweep
    with open(os.path.join(REPO, "tests", "golden", "gemm_sweep_large.json")) as f:
        gold = {(c["case"], c["M"]): c for c in json.load(f)["cases"]}
    int8_peak = 2.0 * peaks.get("bf16_tflops", 1590.0)
    flush = torch.empty(64 << 20, dtype=torch.int32, device="cuda")  # 256 MB > L2
    out_rows = []
    buf = open(model_path(), "rb").read()
    for ci, case in enumerate(sweep.CASES):
        W, m, n = sweep.weights(buf, ci)
        bits_in, f_in, f_out, bits_out = sweep.case_formats(ci)
        N, K = W.shape
        P = bits_in // 8
        plan = _eii.LinearPlan(eng, W, m, n, bits_in, f_in, f_out, bits_out)
        try:
            for M in sweep.MS:
                a = torch.empty((M, K), dtype=torch.int32, device="cuda")
                for b in range(sweep.blocks(M)):
                    blk = sweep.activation_block(ci, M, b, K, bits_in)
                    a[sweep.BLOCK * b:sweep.BLOCK * b + blk.shape[0]].copy_(torch.from_numpy(blk))
                out = torch.empty((M, N), dtype=torch.int32, device="cuda")
                d_out = torch.empty(M, dtype=torch.int64, device="cuda")
                d_acc = torch.empty(M, dtype=torch.int64, device="cuda")
                plan.run(a.data_ptr(), M, out.data_ptr(), N, d_out.data_ptr(), d_acc.data_ptr())
                g = gold.get((ci, M))
                exact = None
                if g is not None:
                    exact = (sweep.hexes(sweep.block_digests(d_acc.cpu().numpy().view(np.uint64), M)) == g["acc_blocks"]
                             and sweep.hexes(sweep.block_digests(d_out.cpu().numpy().view(np.uint64), M)) == g["out_blocks"])
                plan.run(a.data_ptr(), M, out.data_ptr(), N)  # warm-up without digests
                eng.profile_enable(True)
                for _ in range(reps):
                    flush.zero_()
                    plan.run(a.data_ptr(), M, out.data_ptr(), N)
                prof = eng.profile_read()
                eng.profile_enable(False)
                ms, nl = prof["gemm_sweep"]
                t = ms / nl / 1e3
                ops = 2.0 * M * N * K
                tops = ops / t / 1e12
                hbm = (M * K * P + N * K + M * N * 4) / t / 1e9
                out_rows.append({"shape": case[0], "M": M, "N": N, "K": K, "planes": P, "us": round(t * 1e6, 1),
                                 "tops_logical": round(tops, 1), "frac": round(tops / int8_peak, 4),
                                 "tensor_work_frac": round(P * tops / int8_peak, 4),
                                 "hbm_gbs_algorithmic": round(hbm, 1), "exact_vs_reference": exact})
                del a, out, d_out, d_acc
                torch.cuda.empty_cache()
        finally:
            plan.close()
    return {"peak_tops": round(int8_peak, 1),
            "peak_note": "int8 dense = 2 x measured bf16 (MEASURED_PEAKS.json), of measured",
            "ops_note": "tops_logical = 2 M N K / GEMM kernel time; tensor_work_frac counts the byte-plane MMAs "
                        "(planes x logical) against the same peak",
            "path": "eii_linear_plan_run (int32 activations -> byte planes -> tcgen05 kind::i8 GEMM, int32 out)",
            "timing": f"CUDA events around the GEMM launch on the engine's stream, {reps} launches, L2 flushed "
                      "between them", "cases": out_rows}


def run_ours(args):
    import torch
    import _eii
    rank, local, world = rank_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        # the communicator set-up prints "NCCL version ..." on rank 0's stdout, which must carry
        # only the JSON line: point fd 1 at stderr until the first collective has run
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    if rank == 0:
        ensure_model()
    if dist:
        dist.barrier()
    eng = _eii.Engine(model_path(), local)
    s0, ns = shard(rank, world)
    rows = ns * T
    table = token_table()
    ids_host = np.ascontiguousarray(table[s0:s0 + ns, :T])
    ids_dev = torch.from_numpy(ids_host).cuda()
    logits = torch.empty((rows, VOCAB), dtype=torch.int32, device="cuda")
    digests = torch.zeros(ns, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def step():
        eng.forward_device(ids_dev.data_ptr(), ns, T, logits.data_ptr(), VOCAB, digests.data_ptr(), stream)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record()
        for _ in range(args.steps):
            step()
        ev1.record()
        torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    clocks = clk.summary()

    # end to end through the C ABI with host buffers: pinned ids up, digests down, every step
    pinned = torch.from_numpy(ids_host).pin_memory()
    ids_pinned = pinned.numpy()
    dig_host = np.empty(ns, np.uint64)
    import ctypes
    e2e_step = lambda: _eii.check(_eii.lib().eii_forward(eng.h, _eii.ptr(ids_pinned), ns, T, None, None, None,
                                                         _eii.ptr(dig_host)))
    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3)
    barrier()

    # parity: golden subset rows in this shard, and the device digests against the host ones
    with open(os.path.join(REPO, "tests", "golden", "config4_subset.json")) as f:
        sub = json.load(f)
    checked = exact = 0
    for s in sub["sequences"]:
        r = s["row"]
        if s0 <= r < s0 + ns:
            lg = logits[(r - s0) * T:(r - s0 + 1) * T].cpu().numpy()
            checked += 1
            exact += hashlib.sha256(lg.tobytes()).hexdigest() == s["logits_i32_sha256"]
    dig_dev = digests.cpu().numpy().view(np.uint64)
    digest_match = int(np.array_equal(dig_dev, dig_host))
    # per-kernel profile of one more step (not timed above): launches and the dominant kernel
    eng.profile_enable(True)
    step()
    torch.cuda.synchronize()
    prof = {k: v for k, v in eng.profile_read().items() if v[1] > 0}
    eng.profile_enable(False)
    launches_per_step = sum(v[1] for v in prof.values())
    chunk_rows = eng.chunk_sequences(ns, T) * T
    decode = decode_bench(eng, ids_host, ids_dev, ns, digests, stream, barrier, max_over_ranks)
    counts = torch.tensor([checked, exact, digest_match], dtype=torch.int64, device="cuda")
    all_dig = torch.from_numpy(dig_host.view(np.int64).copy()).cuda()
    if dist:
        dist.all_reduce(counts)
        gathered = [torch.empty_like(all_dig) for _ in range(world)]
        dist.all_gather(gathered, all_dig)
        all_dig = torch.cat(gathered)
    if rank == 0:
        tokens = N_SEQ * T
        value = tokens * args.steps / (ms / 1e3)
        e2e_value = tokens * args.steps / (e2e_ms / 1e3)
        peaks = load_peaks()
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 weight x u8/s8 activation planes -> int32 -> int64",
            "data": DATA,
            "config": {"workload": WORKLOAD, "n_seq": N_SEQ, "seq_len": T, "tokens_per_step": tokens,
                       "parallelism": f"dp{world} (sequence shards, no data-path collective)",
                       "chunk_rows": min(chunk_rows, rows),
                       "l2": "no flush needed: each step writes 103 GB of logits and re-reads 135 MB of weights (> 126 MB L2)"},
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": int(N_SEQ * T * 8),
                    "d2h_bytes_per_step": int(N_SEQ * 8),
                    "path": "eii_forward (C ABI) with pinned host ids, per-sequence digests read back"},
            "gpu_launches": int(launches_per_step * args.steps),
            "roofline": roofline(prof, rows, peaks),
            "roofline_hbm": roofline(prof, rows, peaks, kernel="rmsnorm") if "rmsnorm" in prof else None,
            "clocks": clocks,
            "check": {"subset_sequences": int(counts[0]), "subset_exact": int(counts[1]),
                      "digests_device_eq_host_ranks": int(counts[2]),
                      "digest_of_digests": hashlib.sha256(all_dig.cpu().numpy().tobytes()).hexdigest()[:16]},
            "kernels": {k: {"ms": round(v[0], 3), "launches": v[1]} for k, v in prof.items()},
            "decode": dict(decode, value=round(N_SEQ * decode["timed_steps"] / (decode["ms"] / 1e3), 1)),
        }
        if world == 1 and not args.no_cpu_baseline:
            with tempfile.TemporaryDirectory() as td:
                line["cpu_baseline"] = cpu_baseline_from_gpu(eng, model_path(), td)
            line["cpu_baseline_numpy"] = cpu_baseline_numpy(eng, model_path())
        if world == 1 and not args.no_cpu_baseline:
            line["configs_1_3"] = small_configs_bench()
        if world == 1 and not args.no_gemm_sweep:
            del logits
            torch.cuda.empty_cache()
            line["gemm_sweep"] = gemm_sweep_bench(eng, peaks)
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def small_configs_bench(repeat=20):
    """BASELINE configs 1-3 on one GPU: one sequence per forward through eii_forward (the C ABI with
    host buffers: ids up, int32 logits [T, 49152] down), warm, best of `repeat`; each timed forward's
    logits are compared with the sha256 the reference's own exporter wrote (tests/golden)."""
    import _eii
    import synthetic
    out = {}
    for key, name, outlier in (("config1_t24", "t24", False), ("config2_t128", "t128", False),
                               ("config3_t160_outlier", "t160", True)):
        path = model_path()
        if outlier:
            path = os.path.join(MODEL_DIR, "outlier", "model.bin")
            if not os.path.exists(path):
                os.makedirs(os.path.dirname(path), exist_ok=True)
                synthetic.write_model_bin(path, outlier=True)
        with open(os.path.join(REPO, "tests", "golden", f"vectors_{name}.json")) as f:
            golden = json.load(f)
        g = golden
        ids = np.ascontiguousarray(synthetic.token_table()[g["window"], :g["tokens"]][None, :])
        eng = _eii.Engine(path, 0)
        try:
            eng.forward(ids)
            best, exact = None, True
            for _ in range(repeat):
                t0 = time.perf_counter()
                r = eng.forward(ids)
                dt = time.perf_counter() - t0
                best = dt if best is None else min(best, dt)
                exact = exact and hashlib.sha256(r["logits"][0].tobytes()).hexdigest() == \
                    golden["files"]["exp_logits.i32"]["sha256"]
        finally:
            eng.close()
        out[key] = {"T": int(g["tokens"]), "ms": round(best * 1e3, 3), "tokens_per_s": round(g["tokens"] / best, 1),
                    "logits_equal_reference": bool(exact)}
    out["path"] = (f"eii_forward, one sequence, logits copied to host; best of {repeat} warm forwards (wall clock "
                   "around the C call)")
    return out


def run_reference(args):
    rank, local, world = rank_env()
    if rank != 0:
        return
    if not os.path.exists(REF_BIN):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/intref (reference c/intref.c) was not built: "
                                                             "no reference checkout when build() ran"}))
        return
    model = ensure_model()
    procs = cpu_threads()
    with tempfile.TemporaryDirectory() as td:
        dirs = reference_vectors(model, list(range(min(4, procs))), td)
        for _ in range(args.warmup):
            run_reference_c(dirs, procs)
        rates, verdicts = [], []
        t0 = time.time()
        for _ in range(args.steps):
            tps, secs, v, wall = run_reference_c(dirs, procs)
            rates.append(tps)
            verdicts += v
        wall = time.time() - t0
    value = float(np.mean(rates))
    exact = sum("ALL STATES EXACT" in v for v in verdicts)
    cpu = {"value": round(value, 2), "unit": UNIT, "cores": procs, "kind": "reference",
           "sample": f"each step: {procs} sequences x {T} tokens of config 4, one c/intref.c process per host thread"}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * wall / args.steps, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int64 (scalar C)",
        "data": DATA, "config": {"workload": WORKLOAD, "n_seq": N_SEQ, "seq_len": T,
                                 "parallelism": f"{procs} host processes"},
        "cpu_baseline": cpu, "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                                     "d2h_bytes_per_step": 0},
        "check": f"{exact}/{len(verdicts)} reference runs ALL STATES EXACT"}), flush=True)


def run_probe(ns):
    """One forward of the first `ns` config-4 sequences through eii_forward_device (logits and
    digests on the device), for ncu captures of single launches; prints the first digest."""
    import torch
    import _eii
    eng = _eii.Engine(ensure_model(), 0)
    ids = torch.from_numpy(np.ascontiguousarray(token_table()[:ns, :T])).cuda()
    logits = torch.empty((ns * T, VOCAB), dtype=torch.int32, device="cuda")
    digests = torch.zeros(ns, dtype=torch.int64, device="cuda")
    eng.forward_device(ids.data_ptr(), ns, T, logits.data_ptr(), VOCAB, digests.data_ptr(),
                       torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    eng.close()
    print(f"[probe] {ns} x {T} tokens, digest[0] = {int(digests[0].item()) & ((1 << 64) - 1):016x}")


def run_probe_decode(ns):
    """A decoder of `ns` config-4 sequences: a 64-token prompt (eii_decoder_prefill), then four
    single-token steps (eii_decoder_step_device), for ncu captures of the decode attention."""
    import torch
    import _eii
    eng = _eii.Engine(ensure_model(), 0)
    ids = np.ascontiguousarray(token_table()[:ns, :T])
    dec = _eii.Decoder(eng, ns, T)
    dec.prefill(ids[:, :64], logits=False, digests=True)
    ids_t = torch.from_numpy(np.ascontiguousarray(ids[:, 64:68].T)).cuda()
    dig = torch.zeros((4, ns), dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for t in range(4):
        dec.step_device(ids_t[t].data_ptr(), None, VOCAB, dig[t].data_ptr(), stream)
    torch.cuda.synchronize()
    dec.close()
    eng.close()
    print(f"[probe] decode {ns} sequences, position 64..67, digest[0][0] = {int(dig[0, 0].item()) & ((1 << 64) - 1):016x}")


def run_probe_mma():
    """Cycles per tcgen05.mma.kind::i8 (M = 128, K = 32) on every SM: by N alone, and at N = 256 beside
    16 warps of each kind of background work (eii_mma_rate); one JSON object."""
    import _eii
    names = {0: "none", 1: "shared-memory loads", 2: "TMEM loads", 3: "64-bit multiply-add", 4: "global stores",
             5: "32-bit IMAD", 6: "FFMA", 7: "integer ALU", 8: "32x32->64 multiply-accumulate",
             9: "shared-memory stores", 10: "cp.async global->shared", 11: "cp.async.bulk global->shared"}
    peak = 128 * 32 * 256 / 8192.0  # cycles of one N = 256 MMA at 8192 int8 MACs per cycle per SM
    out = {"by_n": {}, "n256_with_16_background_warps": {}}
    for n in (64, 128, 256):
        c = _eii.mma_rate(0, n, 0, 128)
        out["by_n"][n] = {"cycles_per_mma": round(c, 1), "frac_of_8192_macs_per_cycle": round(128 * 32 * n / c / 8192, 3)}
    for z in range(12):
        c = _eii.mma_rate(0, 256, z, 640)
        out["n256_with_16_background_warps"][names[z]] = {"cycles_per_mma": round(c, 1), "frac": round(peak / c, 3)}
    print(json.dumps(out, indent=1))


def run_probe_sweep(spec):
    """One eii_linear_plan_run of sweep case NAME at M rows (spec "NAME:M"), for ncu captures of a
    single GEMM launch; prints the case digest of the outputs."""
    import torch
    import _eii
    import sweep
    name, M = spec.split(":")
    M = int(M)
    ci = [c[0] for c in sweep.CASES].index(name)
    eng = _eii.Engine(ensure_model(), 0)
    W, m, n = sweep.weights(model_path(), ci)
    bits_in, f_in, f_out, bits_out = sweep.case_formats(ci)
    N, K = W.shape
    a = torch.cat([torch.from_numpy(sweep.activation_block(ci, M, b, K, bits_in)) for b in range(sweep.blocks(M))]).cuda()
    out = torch.empty((M, N), dtype=torch.int32, device="cuda")
    d_out = torch.empty(M, dtype=torch.int64, device="cuda")
    plan = _eii.LinearPlan(eng, W, m, n, bits_in, f_in, f_out, bits_out)
    plan.run(a.data_ptr(), M, out.data_ptr(), N, d_out.data_ptr())
    dig = sweep.total(sweep.block_digests(d_out.cpu().numpy().view(np.uint64), M))
    plan.close()
    eng.close()
    print(f"[probe] {name} M={M}: out digest {dig:016x}")


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm-sweep", action="store_true", help="skip the contraction sweep (config 5) at N=1")
    ap.add_argument("--probe", type=int, default=0, metavar="NSEQ",
                    help="profiling target: one untimed forward of NSEQ x 128 tokens on cuda:0, then exit")
    ap.add_argument("--probe-decode", type=int, default=0, metavar="NSEQ",
                    help="profiling target: a 64-token prompt and four decoding steps of NSEQ sequences, then exit")
    ap.add_argument("--probe-mma", action="store_true",
                    help="tcgen05 kind::i8 MMA rate by N and beside background work (eii_mma_rate), then exit")
    ap.add_argument("--probe-sweep", default=None, metavar="NAME:M",
                    help="profiling target: one contraction-sweep GEMM (sweep.py case NAME at M rows), then exit")
    args = ap.parse_args()
    if args.probe:
        run_probe(args.probe)
        return
    if args.probe_sweep:
        run_probe_sweep(args.probe_sweep)
        return
    if args.probe_mma:
        run_probe_mma()
        return
    if args.probe_decode:
        run_probe_decode(args.probe_decode)
        return
    if args.warmup < 3:
        log("[bench] note: fewer than 3 warm-up steps")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
