"""Benchmark of the B200 token sampler on the metric's configuration.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--rows R]

Workload (per GPU): the headline configuration, 1024 rows x 151,936 f32 logits with the
mixed per-row parameters of the benchmark's config 3 (temperature U[0.5,1.5], top_k in
{0,20,40,100}, top_p U[0.8,1.0], repetition penalty U[1.0,1.3] over a 64-token window),
seeded synthetic data.  A step samples every row once through the staged pipeline: seven
launches (tile statistics, per-row prep, tile classification, the exact running sum, the
finish, the big-nucleus stage for top-p rows whose nucleus exceeds a list, then
lrs_sample_rows on the rows the stages leave).  Rows are independent, so N GPUs
run N replicas on different rows (weak scaling, no collective).

value      rows/s over all GPUs with inputs resident in HBM (CUDA events, max over ranks)
e2e        the same metric through the host-buffer entry point (lrs_sample): pinned host
           logits copied in and tokens/statuses copied out inside the timed region
roofline   algorithmic bytes (4 * vocab + 4 * window per row) / step time (the seven launches) vs
           measured HBM copy bandwidth; traffic = DRAM bytes per step from the committed ncu summary
cpu_baseline  the CPU restatement of sampler.rs (oracle) on a bounded sample of the same rows
           (the first --cpu-rows rows, repeated for about --cpu-seconds on all host threads)
--impl reference  times that CPU restatement alone (all host threads) on the same workload
--workload vocab_sharded  config 5 instead: 64 x 151,936 rows whose columns are split over the
           N ranks; a step is the exchange (an NCCL all-to-all of each row's shards to its owner
           rank + row assembly), the owners' sampling and an all-gather of the results; reports
           latency, the exchange's share and bytes, and a check of the tokens against an
           unsharded sample
--workload configs  one GPU, the other configurations of the benchmark at their sizes: config 1
           (one row: latency of a draw through the drop-in single-row API, and 10,000 draws as
           rows sharing the logits), config 2 (greedy), config 3 (mixed, 109,051 wide), config 4
           (nucleus stress, 4096 rows, window 1024); rows/s and the roofline fraction of each
configs    (default run, one GPU; --no-configs skips it) the same configurations 1-4 in brief
           inside the headline line: configs 2-4 at their full sizes on seeded inputs generated
           on the device with the workloads' distributions and parameter mixes (the host
           generator takes minutes at these sizes), config 1 through the drop-in single-row
           API and as 10,000 draws sharing the logits
--workload brief  those brief configurations alone (--configs config4,... picks some;
           --config4-rows sizes config 4 down for profiling)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "llama.rs_b200"))

import numpy as np  # noqa: E402

METRIC = "sampled rows/s at 1024×151,936 f32 logits; % of HBM roofline at 1/2/4/8 GPUs"
WORKLOAD = ("headline: 1024 rows x 151,936 f32 logits per GPU, Gumbel + Zipf-like head under a per-row "
            "permutation, temperature U[0.5,1.5], top_k {0,20,40,100}, top_p U[0.8,1.0], "
            "repetition penalty U[1.0,1.3] over a 64-token window")
FALLBACK_HBM_GBS = 6650.0
STAGE_LAUNCHES = 7  # kernels of one step (the staged pipeline, lrs_stage_launch)
NOMINAL_HBM_GBS = 8000.0  # B200 HBM3e, nominal (the north star quotes 8 TB/s)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name="staged_pipeline_headline.txt", key="dram_bytes_per_step_full_size:"):
    """DRAM bytes per step from the committed ncu summary, if present."""
    path = os.path.join(REPO, "profiles", name)
    try:
        for line in open(path):
            if line.startswith(key):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"lrs_clocks_{os.getpid()}.csv")
        self.window = None

    def start(self):
        """Starts sampling every 20 ms and waits (up to 3 s) for the first sample."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t = time.time()
        while time.time() - t < 3.0:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.01)

    def mark(self, t0, t1):
        """The timed region's wall-clock bounds (samples outside it are dropped)."""
        self.window = (t0, t1)

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.05)
        self.proc.terminate()
        self.proc.wait()
        import datetime
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        samples = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                samples.append((ts, float(f[2]), float(f[3]), f[6:10]))
            except ValueError:
                continue
        if not samples:
            return None
        inside = samples
        if self.window:
            lo, hi = self.window
            inside = [x for x in samples if lo - 0.025 <= x[0] <= hi + 0.025] or samples
        reasons = set()
        for _, _, _, flags in inside:
            for nm, v in zip(names, flags):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": max(x[2] for x in inside),
                "reasons": sorted(reasons), "samples": len(inside)}


def headline_config(rows, vocab, window, world):
    """The `config` object of the headline line, the same for both arms (the reference arm
    samples the same rows of the same workload on the host cores)."""
    return {"workload": WORKLOAD, "rows_per_gpu": rows, "vocab": vocab, "window": window,
            "parallelism": f"rows sharded over {world} GPU(s), replicas, no collective",
            "l2": "inputs larger than L2 (622 MB of logits per GPU per step)"}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


def cpu_sample(w, rows, threads, min_seconds=0.0):
    """Times the CPU restatement on `rows` rows of workload w, repeated until at least
    min_seconds have passed; returns (rows/s, seconds, passes)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O
    O.build()
    sl = slice(0, rows)
    passes = 0
    t = time.perf_counter()
    while True:
        O.sample_batch(w.logits[sl], w.vocab, w.hist[sl], w.hist_len[sl], w.params[sl], w.state[sl],
                       threads=threads)
        passes += 1
        dt = time.perf_counter() - t
        if dt >= min_seconds:
            break
    return rows * passes / dt, dt, passes


def run_reference(args, world, rank):
    """--impl reference: the CPU restatement of sampler.rs on the host cores."""
    if rank != 0:
        return
    from lrs import workloads as W
    rows = args.rows if args.ref_rows is None else min(args.rows, args.ref_rows)
    w = W.headline(row_ids=range(rows))
    threads = os.cpu_count() or 1
    times = []
    for i in range(args.warmup + args.steps):
        _, dt, _ = cpu_sample(w, rows, threads)
        if i >= args.warmup:
            times.append(dt)
    value = rows * len(times) / sum(times)
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": headline_config(rows, w.vocab, w.window, world),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} rows of the headline workload per step, one sampler per row, "
                                   f"rows spread over {threads} host threads"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_vocab_sharded(args, world, rank, local):
    """Config 5: columns split over the ranks; each row sampled by its owner rank (lrs.sharded)."""
    import datetime

    import torch
    import torch.distributed as dist

    import lrs
    from lrs import sharded
    from lrs import workloads as W
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    w = W.vocab_sharded()
    rows, V = w.rows, w.vocab
    cols = sharded.shard_columns(V, world, rank)
    vsamp = sharded.VocabShardedSampler(rows, V, w.window, device=local)
    shard = torch.from_numpy(np.ascontiguousarray(w.logits[:, cols])).to(dev)
    hist = torch.from_numpy(w.hist.view(np.int32)).to(dev)
    hlen = torch.from_numpy(w.hist_len.view(np.int32)).to(dev)
    params = torch.from_numpy(w.params.view(np.uint8)).to(dev)
    state0 = torch.from_numpy(w.state.view(np.int64)).to(dev)
    state = state0.clone()
    tokens = torch.zeros(rows, dtype=torch.int32, device=dev)
    status = torch.zeros(rows, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    # correctness first: one step from the initial states against an unsharded sample
    vsamp.sample(shard, params, state, tokens, hist=hist, hist_len=hlen, status=status)
    torch.cuda.synchronize()
    ok = None
    if rank == 0:
        ref = lrs.BatchSampler(rows, V, w.window, device=local)
        full = torch.from_numpy(w.logits).to(dev)
        st2 = state0.clone()
        tok2 = torch.zeros(rows, dtype=torch.int32, device=dev)
        ref.sample_device(full, params, st2, tok2, hist=hist, hist_len=hlen)
        torch.cuda.synchronize()
        ok = bool(torch.equal(tok2, tokens)) and bool(torch.equal(st2, state)) and int((status != 0).sum()) == 0
        ref.close()
    for _ in range(args.warmup):
        vsamp.sample(shard, params, state, tokens, hist=hist, hist_len=hlen, status=status)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ex = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        ex[i][0].record(stream)
        vsamp.exchange(shard)
        ex[i][1].record(stream)
        vsamp.sample_owned(params, state, tokens, hist=hist, hist_len=hlen, status=status)
    t1.record(stream)
    torch.cuda.synchronize()
    total_ms = t0.elapsed_time(t1)
    exch_ms = sum(a.elapsed_time(b) for a, b in ex)
    if world > 1:
        tt = torch.tensor([total_ms, exch_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms, exch_ms = float(tt[0].item()), float(tt[1].item())
    if rank == 0:
        line = {
            "metric": "config 5 (vocab-sharded) step latency", "value": total_ms / args.steps, "unit": "ms",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"config 5: {rows} x {V} f32 rows, columns split over {world} GPU(s) "
                                   f"({V // world} each), top_k 50, top_p 0.95, temp 0.7",
                       "parallelism": f"vocabulary over {world} GPU(s); row r sampled by the rank owning its "
                                      f"row block: one all-to-all of the shards to the owners, one all-gather "
                                      f"of the results"},
            "exchange_ms_per_step": exch_ms / args.steps, "exchange_share": exch_ms / total_ms,
            "exchange_bytes_per_rank": vsamp.exchange_bytes(),
            "all_gather_bytes_per_rank": (world - 1) * rows * (V // world) * 4,
            "tokens_match_unsharded": ok,
            "gpu_launches": (1 + STAGE_LAUNCHES) * args.steps,  # the row assembly, then the sampler
        }
        print(json.dumps(line), flush=True)
    vsamp.close()
    if world > 1:
        dist.destroy_process_group()


def run_configs(args):
    """The benchmark's configurations 1-4 on one GPU (auxiliary to the headline line)."""
    import torch
    import lrs
    from lrs import workloads as W
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, _ = peaks()
    out = {"metric": "configs 1-4 of the benchmark (auxiliary)", "n_gpus": 1, "data": "synthetic", "configs": {}}

    def device_rate(w, shared_row=False, reps=None):
        rows = len(w.params)
        bs = lrs.BatchSampler(rows, w.vocab, max(w.window, 1))
        # (shared_row: every row reads logits row 0, ld = 0)
        x = torch.from_numpy(w.logits).to(dev)
        hist = torch.from_numpy(w.hist.view(np.int32)).to(dev) if w.window else None
        hlen = torch.from_numpy(w.hist_len.view(np.int32)).to(dev) if w.window else None
        params = torch.from_numpy(w.params.view(np.uint8)).to(dev)
        state = torch.from_numpy(w.state.view(np.int64)).to(dev)
        tokens = torch.zeros(rows, dtype=torch.int32, device=dev)
        status = torch.zeros(rows, dtype=torch.int32, device=dev)
        ld = 0 if shared_row else None

        def step():
            bs.sample_device(x, params, state, tokens, n=w.vocab, hist=hist, hist_len=hlen, status=status, ld=ld,
                             rows=rows)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        if int((status != 0).sum()):
            raise SystemExit("a row reported a non-zero status")
        k = reps or max(3, args.steps // 2)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k):
            step()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / k
        bs.close()
        row_bytes = 4 * w.vocab * (0 if shared_row else 1) + 4 * w.window
        frac = (rows * row_bytes / (ms / 1e3) / 1e9) / peak if row_bytes else None
        return {"rows": rows, "vocab": w.vocab, "window": w.window, "ms_per_step": ms,
                "rows_per_s": rows / (ms / 1e3), "roofline_frac": frac}

    c = out["configs"]
    c["config2_greedy"] = device_rate(W.greedy())
    c["config3_mixed"] = device_rate(W.mixed())
    c["config4_nucleus"] = device_rate(W.nucleus(), reps=3)
    # config 1: 10,000 draws on one row's logits and history (per-draw PRNG states)
    w1 = W.single(1)
    draws = 10000

    class Draws:  # one logits row, `draws` rows of parameters, history and PRNG states
        vocab, window = w1.vocab, w1.window
        logits = w1.logits[:1]
        params = np.repeat(w1.params, draws)
        hist = np.repeat(w1.hist, draws, axis=0)
        hist_len = np.repeat(w1.hist_len, draws)
        state = W.xorshift_states(int(w1.state[0]), draws)

    c["config1_batched_draws"] = device_rate(Draws, shared_row=True, reps=5)
    # config 1: one draw at a time through the drop-in Sampler (host logits, synchronous)
    s = lrs.Sampler(42)
    sp = lrs.SamplingParams(temperature=float(w1.params["temperature"][0]), top_k=int(w1.params["top_k"][0]),
                            top_p=float(w1.params["top_p"][0]),
                            repetition_penalty=float(w1.params["repetition_penalty"][0]),
                            repeat_last_n=int(w1.params["repeat_last_n"][0]), seed=42)
    recent = w1.hist[0, :int(w1.hist_len[0])]
    for _ in range(5):
        s.sample(w1.logits[0], sp, recent)
    n1 = 200
    t = time.perf_counter()
    for _ in range(n1):
        s.sample(w1.logits[0], sp, recent)
    us = (time.perf_counter() - t) / n1 * 1e6
    c["config1_single_draw"] = {"us_per_draw": us, "api": "lrs_sampler_sample (host logits, synchronous)"}
    print(json.dumps(out), flush=True)


def brief_configs(dev, peak, only=None, rows4=4096):
    """Configs 1-4 in brief for the headline line (one GPU): configs 2-4 at their full sizes on
    seeded inputs generated on the device with the distributions and parameter mixes of
    lrs.workloads (greedy rows with planted ties; Zipf-like rows under a per-row permutation
    with the mixed parameters; flat and spiked nucleus-stress rows with a 1,024-token window),
    config 1 on the workload's own row: one draw at a time through the drop-in single-row API,
    and 10,000 draws as rows sharing the logits.  rows/s and the roofline fraction of each.
    only: the configurations to run (config1 .. config4; None: all); rows4: config 4's rows."""
    import torch
    import lrs
    from lrs import workloads as W
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242)
    rng = np.random.default_rng(4242)

    def timed(x, params, window, reps, ld=None, rows=None, state=None):
        rows = rows if rows is not None else x.shape[0]
        V = x.shape[1]
        bs = lrs.BatchSampler(rows, V, max(window, 1))
        P = torch.from_numpy(np.ascontiguousarray(params).view(np.uint8)).to(dev)
        if state is None:
            state = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
        st = torch.from_numpy(state.view(np.int64)).to(dev)
        hist = hl = None
        if window:
            hist = torch.randint(0, V, (rows, window), device=dev, generator=gen, dtype=torch.int32)
            hl = torch.full((rows,), window, dtype=torch.int32, device=dev)
        tok = torch.zeros(rows, dtype=torch.int32, device=dev)
        sts = torch.zeros(rows, dtype=torch.int32, device=dev)

        def step():
            bs.sample_device(x, P, st, tok, n=V, hist=hist, hist_len=hl, status=sts, ld=ld, rows=rows)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        if int((sts != 0).sum()):
            raise SystemExit("a row reported a non-zero status")
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            step()
        b.record()
        torch.cuda.synchronize()
        bs.close()
        ms = a.elapsed_time(b) / reps
        row_bytes = 4 * V * (0 if ld == 0 else 1) + 4 * window
        return {"rows": rows, "vocab": V, "window": window, "ms_per_step": ms, "rows_per_s": rows / (ms / 1e3),
                "roofline_frac": (rows * row_bytes / (ms / 1e3) / 1e9) / peak}

    def params(rows, t, k, p, pen, last):
        out = np.zeros(rows, lrs.PARAMS_DTYPE)
        out["temperature"], out["top_k"], out["top_p"] = t, k, p
        out["repetition_penalty"], out["repeat_last_n"] = pen, last
        return out

    res = {"data": "configs 2-4: seeded inputs generated on the device with the distributions and parameter "
                   "mixes of lrs.workloads; config 1: the workload's own row"}
    V = W.QWEN_VOCAB
    want = (lambda c: only is None or c in only)
    # config 2: 256 greedy rows, the max planted at 2-4 positions in 10% of them
    if want("config2"):
        x = torch.randn(256, V, device=dev, generator=gen) * 3.0
        for r in range(3, 256, 10):
            k = int(rng.integers(2, 5))
            pos = torch.randperm(V, device=dev, generator=gen)[:k]
            x[r, pos] = x[r].max() + abs(float(rng.standard_normal())) + 0.5
        res["config2_greedy"] = timed(x, params(256, 0.0, 0, 1.0, 1.0, 64), 0, 20)
        del x
    # config 3: 1024 x 109,051, Gumbel + 2 log(1/rank^1.1) under a per-row permutation, mixed parameters
    if want("config3"):
        Vp = W.PRUNED_VOCAB
        u = torch.rand(1024, Vp, device=dev, generator=gen).clamp_(1e-12, 1.0 - 1e-7)
        head = -2.2 * torch.log(torch.arange(1, Vp + 1, device=dev, dtype=torch.float64)).float()
        perm = torch.argsort(torch.rand(1024, Vp, device=dev, generator=gen), dim=1)
        x = (-torch.log(-torch.log(u)) + head[perm]).contiguous()
        del u, perm
        p3 = params(1024, 1.0, 0, 1.0, 1.0, 64)
        p3["temperature"] = rng.uniform(0.5, 1.5, 1024)
        p3["top_k"] = np.array([0, 20, 40, 100])[rng.integers(0, 4, 1024)]
        p3["top_p"] = rng.uniform(0.8, 1.0, 1024)
        p3["repetition_penalty"] = rng.uniform(1.0, 1.3, 1024)
        res["config3_mixed"] = timed(x, p3, 64, 20)
        del x
    # config 4: 4096 x 151,936, even rows flat N(0, 0.5), odd rows N(0, 2) with +12 on one index
    if want("config4"):
        x = torch.randn(rows4, V, device=dev, generator=gen)
        x[0::2] *= 0.5
        x[1::2] *= 2.0
        spikes = torch.randint(0, V, (rows4 // 2,), device=dev, generator=gen)
        x[torch.arange(1, rows4, 2, device=dev), spikes] += 12.0
        res["config4_nucleus"] = timed(x, params(rows4, 1.0, 0, 0.9, 1.2, 1024), 1024, 5)
        del x
    torch.cuda.empty_cache()
    if not want("config1"):
        return res
    # config 1: the single row, 10,000 draws as rows sharing the logits (ld = 0), and one draw at
    # a time through the drop-in Sampler (host logits, one synchronous round trip a draw)
    w1 = W.single(1)
    draws = 10000
    x = torch.from_numpy(w1.logits).to(dev)
    p1 = np.repeat(w1.params, draws)
    res["config1_batched_draws"] = timed(x, p1, w1.window, 5, ld=0, rows=draws,
                                         state=W.xorshift_states(int(w1.state[0]), draws))
    s = lrs.Sampler(42)
    sp = lrs.SamplingParams(temperature=float(w1.params["temperature"][0]), top_k=int(w1.params["top_k"][0]),
                            top_p=float(w1.params["top_p"][0]),
                            repetition_penalty=float(w1.params["repetition_penalty"][0]),
                            repeat_last_n=int(w1.params["repeat_last_n"][0]), seed=42)
    recent = w1.hist[0, :int(w1.hist_len[0])]
    for _ in range(5):
        s.sample(w1.logits[0], sp, recent)
    n1 = 200
    t = time.perf_counter()
    for _ in range(n1):
        s.sample(w1.logits[0], sp, recent)
    res["config1_single_draw"] = {"us_per_draw": (time.perf_counter() - t) / n1 * 1e6,
                                  "api": "lrs_sampler_sample (host logits, synchronous)"}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--rows", type=int, default=1024)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-rows", type=int, default=1024)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="cpu_baseline: repeat the sample this long")
    ap.add_argument("--ref-rows", type=int, default=None,
                    help="--impl reference: rows per step (default: --rows, the GPU arm's rows)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg (profiling runs)")
    ap.add_argument("--no-configs", action="store_true", help="skip the brief configs 1-4 in the headline line")
    ap.add_argument("--workload", default="headline", choices=["headline", "vocab_sharded", "configs", "brief"])
    ap.add_argument("--configs", default=None, help="--workload brief: comma list of config1..config4 (default all)")
    ap.add_argument("--config4-rows", type=int, default=4096, help="--workload brief: rows of config 4")
    args = ap.parse_args()
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.workload == "vocab_sharded":
        run_vocab_sharded(args, world, rank, local)
        return
    if args.workload == "configs":
        if rank == 0:
            run_configs(args)
        return
    if args.workload == "brief":
        if rank == 0:
            import torch
            torch.cuda.set_device(0)
            only = set(args.configs.split(",")) if args.configs else None
            print(json.dumps(brief_configs(torch.device("cuda", 0), peaks()[0], only, args.config4_rows)), flush=True)
        return

    import torch
    import lrs
    from lrs import workloads as W
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist

    rows = args.rows
    w = W.headline(row_ids=range(rank * rows, (rank + 1) * rows))
    V, Wn = w.vocab, w.window
    bs = lrs.BatchSampler(rows, V, Wn, device=local)
    logits = torch.from_numpy(w.logits).to(dev)
    hist = torch.from_numpy(w.hist.view(np.int32)).to(dev)
    hlen = torch.from_numpy(w.hist_len.view(np.int32)).to(dev)
    params = torch.from_numpy(w.params.view(np.uint8)).to(dev)
    state = torch.from_numpy(w.state.view(np.int64)).to(dev)
    tokens = torch.zeros(rows, dtype=torch.int32, device=dev)
    status = torch.zeros(rows, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        bs.sample_device(logits, params, state, tokens, n=V, hist=hist, hist_len=hlen, status=status,
                         stream=stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    bad = int((status != 0).sum())
    if bad:
        raise SystemExit(f"{bad} rows reported a non-zero status")

    # (rank 0 alone samples clocks: its line is the one printed, and a sampler per rank adds
    # driver queries every 20 ms on every GPU during a timed region of a few tens of ms)
    clocks = Clocks(local) if rank == 0 else None
    if clocks:
        clocks.start()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    w0 = time.time()
    t0.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.mark(w0, time.time())
    if pg:
        pg.barrier()
    clk = clocks.stop() if clocks else None
    total_ms = t0.elapsed_time(t1)
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    if pg:
        tt = torch.tensor([total_ms], device=dev)
        pg.all_reduce(tt, op=pg.ReduceOp.MAX)
        total_ms = float(tt.item())
    value = world * rows * args.steps / (total_ms / 1000.0)

    # e2e: host buffers through lrs_sample (pinned logits, synchronous call)
    pinned = torch.from_numpy(w.logits).pin_memory()
    host_logits = pinned.numpy()
    bs.set_params(w.params)
    bs.set_state(w.state)
    bs.sample(host_logits, hist=w.hist, hist_len=w.hist_len)  # warm
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    te = time.perf_counter()
    for _ in range(args.e2e_steps):
        bs.sample(host_logits, hist=w.hist, hist_len=w.hist_len)
    e2e_s = time.perf_counter() - te
    if pg:
        tt = torch.tensor([e2e_s], device=dev)
        pg.all_reduce(tt, op=pg.ReduceOp.MAX)
        e2e_s = float(tt.item())
    e2e_value = world * rows * args.e2e_steps / e2e_s
    h2d = rows * V * 4 + rows * Wn * 4 + rows * 4
    d2h = rows * 4 * 2

    bytes_per_row = 4 * V + 4 * Wn
    mean_launch = statistics.mean(launch_ms)
    achieved = rows * bytes_per_row / (mean_launch / 1000.0) / 1e9
    peak, kind = peaks()
    traffic = profile_traffic()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        nrows = min(args.cpu_rows, rows)
        v, dt, passes = cpu_sample(w, nrows, threads, args.cpu_seconds)
        # the reference's sampler is single-threaded: the same sample on one host thread too
        n1 = min(nrows, 64)
        v1, dt1, _ = cpu_sample(w, n1, 1, 0.0)
        cpu = {"value": v, "unit": "rows/s", "cores": threads, "kind": "port",
               "sample": f"first {nrows} rows of this rank's headline workload, {passes} passes, one sampler "
                         f"per row over {threads} host threads ({dt:.1f} s)",
               "value_1_thread": v1, "sample_1_thread": f"first {n1} rows on one host thread ({dt1:.1f} s)"}

    aux = None
    if rank == 0 and world == 1 and not args.no_configs:
        bs.close()
        bs = None
        del logits
        torch.cuda.empty_cache()
        aux = brief_configs(dev, peak)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": headline_config(rows, V, Wn, world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "nominal_peak": NOMINAL_HBM_GBS, "frac_of_nominal": achieved / NOMINAL_HBM_GBS,
                         "peak_kind": kind,
                         "kernel": "staged pipeline: lrs_stage_stats, _prep, _classify, _sum, _finish, _big, "
                                   "lrs_sample_rows",
                         "kernel_ms_mean": mean_launch, "bytes_per_launch": rows * bytes_per_row},
            "e2e": {"value": e2e_value, "unit": "rows/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": STAGE_LAUNCHES * args.steps,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        if aux is not None:
            line["configs"] = aux
        print(json.dumps(line), flush=True)
    if bs is not None:
        bs.close()
    if pg:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
