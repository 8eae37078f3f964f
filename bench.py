"""Benchmark of the hot path: MiniCPM-4 backbone decode on B200 (BASELINE.json config 2 at N=1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step is one decode step of the 0.5B-shaped bf16 stack (24 layers, hidden 1024, 16/2 heads,
FFN 4096) at batch 1, for a request whose 512-position prefill ran first; positions advance from
512 each step. `value` is decode tokens/s over all ranks, timed with CUDA events on the runtime's
stream with inputs resident in HBM; `e2e` is the same through the C-ABI step with host buffers
(tg_decoder_step_rows: host-to-device copy of x and the placement, device-to-host read of the
output, every step). The weights (717 MB) are far larger than the 126 MB L2, so no flush is
needed between steps.

Under torchrun (N > 1) each rank holds a full replica and decodes its own request (the path
shards by request: no collective on the data path); the job's time is the max over ranks. At N > 1
the line also carries config 5, the request-sharded serving BASELINE names for 1/2/4/8 GPUs
(`extras.serve_c5`: aggregate tokens/s, p50/p99 step latency, each rank's busy time).

`roofline` is the decode step's: its algorithmic bytes (every weight once, the KV positions read)
over its measured time against MEASURED_PEAKS.json's HBM rate; with the persistent step (the
default at batch 1) the step is one launch, and `traffic` is that launch's DRAM bytes as the
committed ncu summary under profiles/ records them.

`--impl reference` times the reference's CPU path for the same workload: tgtts-v4 itself cannot
run here (Rust toolchain absent; its GPU path is Vulkan), so it is the C restatement under
oracle/, on all host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PREFILL = 512
CAPACITY = 1024
METRIC = "LM decode tokens/s (0.5B-shaped bf16 backbone, batch 1, position 512+)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="skip the prefill/GEMM side measurements")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--workload", default="decode", choices=["decode", "serve", "sweep", "gemm", "local"],
                    help="decode: config 2 (the headline line); serve: config 5, request-sharded "
                         "serving; sweep: decode step time by batch rows; gemm: config 4's four "
                         "projection GEMMs alone; local: VoxCPM2's patch sampler and local encoder")
    ap.add_argument("--rows", type=int, default=32768, help="gemm: rows (M)")
    ap.add_argument("--sweep-rows", default="1,16,64,128", help="sweep: the decoders' rows, comma-separated")
    ap.add_argument("--requests", type=int, default=2048, help="serve: requests over all GPUs")
    return ap.parse_args()


def dist_init(n):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class Clocks:
    """nvidia-smi samples of this GPU's clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"tg_clocks_{os.getpid()}_{device}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100", "-f", str(self.path)],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            try:
                self.lines = [l for l in self.path.read_text().splitlines() if l.strip()]
                self.path.unlink()
            except OSError:
                pass

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def kv_bytes(shape, position, bytes_per_value=2):
    """The keys and values a decode step at `position` reads over every layer: positions
    0 .. position exactly (the algorithmic bytes; past a row's position the kernels read nothing)."""
    return shape.layers * 2 * shape.kv_heads * (position + 1) * shape.head_dim * bytes_per_value


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def sustained_tflops():
    """MEASURED_PEAKS.json's sustained bf16 rate (a seconds-long GEMM loop under the power cap): the
    denominator for kernels timed inside a long program, such as the prefill's GEMMs."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()).get("bf16_tflops_sustained")
    return None


def stream_ctx(ctx):
    import torch

    return torch.cuda.ExternalStream(ctx.stream, device=f"cuda:{ctx.device}")


def run_ours(args, rank, world, local):
    import torch

    import __graft_entry__ as entry

    pkg = entry.load_package()
    from tgtts_v4_b200 import synthetic as syn

    torch.cuda.set_device(local)
    ctx = pkg.Context(local)
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=CAPACITY)
    weights = syn.make_weights(cfg, seed=0, as_bits=True)
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="bf16")
    dec.load(weights)
    pre = pkg.Prefill(dec, max_rows=PREFILL)
    x0 = syn.make_inputs(PREFILL, cfg.hidden, seed=1 + rank, bf16=True)
    pre_out = pre.run(0, x0)
    stream = stream_ctx(ctx)
    H = cfg.hidden

    # ---- value: device-resident decode steps, CUDA events on the runtime's stream ----
    x_dev = torch.from_numpy(pre_out[-1:].copy()).to(f"cuda:{local}")
    out_dev = torch.empty_like(x_dev)
    torch.cuda.synchronize()

    def positions(i):
        return PREFILL + (i % (CAPACITY - PREFILL))

    clocks = Clocks(local)
    clocks.__enter__()
    for i in range(args.warmup):
        dec.step_device([positions(i)], x_dev.data_ptr(), out_dev.data_ptr())
    ctx.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        dec.step_device([positions(args.warmup + i)], x_dev.data_ptr(), out_dev.data_ptr())
    e1.record(stream)
    e1.synchronize()
    ctx.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms, world)
    ms_per_step = ms_max / args.steps
    value = world * args.steps / (ms_max / 1e3)

    # ---- e2e: the C-ABI step with host buffers, every step's copies inside the timed region ----
    x_host = pre_out[-1:].copy()
    for i in range(min(args.warmup, 5)):
        dec.step_rows([pkg.Row(positions(i), 0)], x_host)
    barrier(world)
    t0 = time.perf_counter()
    for i in range(args.steps):
        dec.step_rows([pkg.Row(positions(args.warmup + i), 0)], x_host)
    t_e2e = time.perf_counter() - t0
    clocks.__exit__(None, None, None)
    t_e2e = max_over_ranks(t_e2e, world)
    e2e = world * args.steps / t_e2e

    result = None
    extras = {}
    labels = dec.labels()
    # Config 5 (request-sharded serving) on the same GPUs: at N > 1 every rank takes part.
    if world > 1 and not args.no_extras:
        extras["serve_c5"] = serve_config5(pkg, syn, ctx, torch, rank, world, local, args.requests, weights)
    if rank == 0:
        hbm, tc, peak_kind = peaks()
        # The steps timed ran from position PREFILL; a step at position p reads p + 1 positions.
        mean_pos = PREFILL + (args.warmup + (args.steps - 1) / 2.0)
        step_bytes = shape.weight_bytes(2) + kv_bytes(shape, int(round(mean_pos)))
        roof = step_roofline(labels, step_bytes, ms_per_step, hbm, peak_kind)
        if not args.no_extras and world == 1:
            extras["gemv_gate_up_alone"] = gate_up_roofline(pkg, ctx, shape, stream, torch, hbm, peak_kind)
        # The side measurements and the CPU baseline are single-GPU numbers: at N > 1 they would
        # only hold the other GPUs.
        if not args.no_extras and world == 1:
            extras.update(side_measurements(pkg, syn, ctx, torch, tc, peak_kind, weights))
        cpu = None if args.no_cpu or world > 1 else cpu_baseline(syn, shape, weights)
        c = clocks.summary()
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,0.02) weights seed 0 (numpy PCG64), N(0,1) bf16 embeddings",
            "config": {"workload": "config 2: 0.5B-shaped bf16 backbone, 512-position prefill then "
                                   "decode at batch 1, one request per GPU",
                       "layers": 24, "hidden": 1024, "heads": "16q/2kv", "head_dim": 64, "ffn": 4096,
                       "batch": 1, "positions": f"{PREFILL}..", "parallelism": f"replicas x{world}",
                       "l2": "weights 717 MB > 126 MB L2 each step; no flush"},
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": H * 4 + 4,
                    "d2h_bytes_per_step": H * 4},
            "roofline": roof,
            "cpu_baseline": cpu,
            "gpu_launches": len(labels) * args.steps,
            "clocks": {"sm_mhz": c["sm_mhz"], "sm_max_mhz": c["sm_max_mhz"], "reasons": c["reasons"]},
            "extras": extras,
        }
    pre.close()
    dec.close()
    ctx.close()
    return result


STEP_PROFILE = ROOT / "profiles" / "decode_step_persistent_config2.md"


def profiled_traffic(path):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) as the committed ncu
    summary `path` records them on its line "dram bytes per launch: N", with the summary's name;
    None when there is no such summary. The summary is re-captured whenever the kernel changes."""
    try:
        for line in path.read_text().splitlines():
            if line.lower().startswith("dram bytes per launch:"):
                return int(line.split(":", 1)[1].strip().replace(",", "")), str(path.relative_to(ROOT))
    except (OSError, ValueError):
        pass
    return None, None


def step_roofline(labels, step_bytes, ms_per_step, hbm, peak_kind):
    """The decode step against HBM: its algorithmic bytes (every weight once, the KV positions the
    steps read) over its measured time. With the persistent step the whole step is one launch, so the
    step is the dominant kernel; with six kernels a layer it names the chain."""
    persistent = labels == ["decode_step"]
    achieved = step_bytes / (ms_per_step * 1e6)
    traffic, source = profiled_traffic(STEP_PROFILE) if persistent else (None, None)
    return {"kernel": "decode_step (persistent: the whole step, 24 layers, in one launch)" if persistent
            else f"the step's {len(labels)}-kernel chain",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved / hbm, 4), "traffic": traffic,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)", "bytes_per_launch": step_bytes,
            "launch_us": round(ms_per_step * 1e3, 2),
            "traffic_source": (f"{source}: ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch"
                               if source else None),
            "how": "bytes = every weight once + the KV positions read; time = the timed steps' CUDA events"}


def gate_up_roofline(pkg, ctx, shape, stream, torch, hbm, peak_kind, layers=24, reps=20):
    """The dominant decode kernel, gemv_gate_up (56% of a step's weight bytes), timed alone: a
    program of one launch per layer over `layers` distinct weight buffers (403 MB, beyond L2), as
    the decode step chains them, timed with CUDA events on the runtime's stream. Algorithmic bytes
    per launch: the 2 I H bf16 weights, the f32 input row and the f32 output row."""
    H, I = shape.hidden, shape.inner
    wbytes = 2 * I * H * 2
    x = pkg.Memory(ctx, H * 4)
    x.write(np.random.default_rng(0).standard_normal(H, dtype=np.float32))
    g = pkg.Memory(ctx, H * 4)
    g.write(np.ones(H, np.float32))
    w = pkg.Memory(ctx, layers * wbytes)
    w.fill(0x3C003C00)  # bf16 pairs of 0.0078125
    out = pkg.Memory(ctx, I * 4)
    p = pkg.params(shape, "bf16", rows=1)
    n = layers * reps
    prog = pkg.Program(ctx, [("gemv_gate_up", p, [(x, 0, H * 4), (g, 0, H * 4), (w, (i % layers) * wbytes, wbytes),
                                                   (out, 0, I * 4)], f"gate_up.{i}") for i in range(n)])
    for _ in range(3):
        prog.run()
    prog.run()
    ns = prog.elapsed_ns() / n  # the program's own start and end events on the runtime's stream
    algo = wbytes + H * 4 + I * 4
    achieved = algo / ns
    prog.close()
    return {"kernel": "gemv_gate_up (fused RMSNorm + gate/up GEMV + SiLU-mul), batch 1", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)", "bytes_per_launch": algo,
            "launch_us": round(ns / 1e3, 3), "traffic": None,
            "how": f"one program of {n} back-to-back launches cycling over {layers} distinct weight buffers, "
                   "CUDA events at its ends"}


def side_measurements(pkg, syn, ctx, torch, tc_peak, peak_kind, weights):
    """Prefill throughput (config 2's 512-position prefill, and config 4's 16 x 2048) and the
    tcgen05 GEMM's tensor-core fraction on config 4's gate/up projection."""
    out = {}
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=2048)
    dec = pkg.Decoder(ctx, shape, rows=16, slots=16, dtype="bf16")
    dec.load(weights)
    rows = 16 * 2048
    x = torch.randn(rows, cfg.hidden, device=f"cuda:{ctx.device}").to(torch.bfloat16).float()
    o = torch.empty_like(x)
    runs = [(0, 2048, s) for s in range(16)]
    # The prefill's time from a program recorded without per-dispatch events (events between the
    # dispatches would keep each kernel from starting under the one before); its shares from one
    # recorded with them.
    plain = pkg.Prefill(dec, max_rows=rows)
    plain.run_batch_device(runs, x.data_ptr(), o.data_ptr())
    ctx.synchronize()
    times = []
    for _ in range(3):
        plain.run_batch_device(runs, x.data_ptr(), o.data_ptr())
        ctx.synchronize()
        times.append(plain.elapsed_ns())
    plain.close()
    pre = pkg.Prefill(dec, max_rows=rows, timed=True)
    pre.run_batch_device(runs, x.data_ptr(), o.data_ptr())
    ctx.synchronize()
    per = {}
    for _ in range(3):
        pre.run_batch_device(runs, x.data_ptr(), o.data_ptr())
        ctx.synchronize()
        for label, ns in pre.timings():
            per[label] = per.get(label, 0.0) + ns / 3
    ns = min(times)
    gemm_flops = 2 * rows * 14_942_208 * 24
    gemm_ns = sum(v for k, v in per.items() if k.endswith("_proj"))
    gu_ns = per.get("gate_up_proj", 0.0)
    gu_flops = 2 * rows * 8192 * 1024 * 24
    # Causal attention: S = q k^T and P v over each row's positions 0..p, 2 x 2 x (p + 1) x hd
    # flops a head a row, summed over the runs' rows: 2 x S (S + 1) x hd x heads a run a layer.
    att_ns = per.get("attention_rows", 0.0)
    att_flops = 2 * 2048 * 2049 * cfg.head_dim * cfg.heads * 16 * 24
    out["prefill_c4"] = {"rows": rows, "tokens_per_s": round(rows / (ns / 1e9), 1), "ms": round(ns / 1e6, 3),
                         "gemm_tflops": round(gemm_flops / gemm_ns / 1e3, 1),
                         "gemm_frac_of_peak": round(gemm_flops / gemm_ns / 1e3 / tc_peak, 4),
                         "gemm_frac_of_sustained_peak": (round(gemm_flops / gemm_ns / 1e3 / sustained_tflops(), 4)
                                                         if sustained_tflops() else None),
                         "gate_up_gemm_tflops": round(gu_flops / gu_ns / 1e3, 1),
                         "attention_tflops": round(att_flops / att_ns / 1e3, 1) if att_ns else None,
                         "attention_frac_of_peak": round(att_flops / att_ns / 1e3 / tc_peak, 4) if att_ns else None,
                         "peak_tflops": tc_peak, "peak_source": peak_kind,
                         "share": {k: round(v / sum(per.values()), 4) for k, v in sorted(per.items(), key=lambda kv: -kv[1])}}
    pre.close()
    dec.close()
    out["decode_c3"] = continuous_c3(pkg, syn, ctx, torch, weights)
    out["logits_head"] = logits_head(pkg, syn, ctx)
    return out


def logits_head(pkg, syn, ctx, vocab=32000, reps=99):
    """The optional vocabulary head at batch 1 (gemv_linear, bf16 W [32000][1024], 65.5 MB): three
    heads' weights (197 MB, past L2) taken in turn, `reps` launches in one program, CUDA events at
    its ends."""
    from tgtts_v4_b200.lm_side import LogitsHead

    hbm, _, _ = peaks()
    H = syn.S05B.hidden
    heads = []
    for i in range(3):
        head = LogitsHead(pkg, ctx, H, vocab, rows=1)
        head.load(np.random.default_rng(i).standard_normal((vocab, H), dtype=np.float32) * np.float32(0.02))
        head(np.ones((1, H), np.float32))
        heads.append(head)
    prog = pkg.Program(ctx, [heads[i % 3].dispatch for i in range(reps)])
    prog.run()
    prog.run()
    us = prog.elapsed_ns() / reps / 1e3
    gbs = vocab * H * 2 / (us * 1e3)
    prog.close()
    return {"vocab": vocab, "hidden": H, "rows": 1, "us": round(us, 2), "weight_gbs": round(gbs, 1),
            "frac_of_hbm": round(gbs / hbm, 4)}


def continuous_c3(pkg, syn, ctx, torch, weights, steps=300, check=8, slots=64):
    """Config 3: 64 requests under continuous batching (contexts uniform 64-2048, seed 2; each
    finishes after uniform 32-512 steps and is replaced by a request with a fresh 128-position
    prompt), `steps` decode steps with the refills' prefills between them, timed with CUDA events
    on the runtime's stream (device time from the first step to the last, host gaps included). The
    same schedule again with every step's outputs read to the host (e2e); then `check` requests that
    ran start to finish are re-run alone through the same server and compared bit for bit."""
    from tgtts_v4_b200 import serving

    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=2560)
    dec = pkg.Decoder(ctx, shape, rows=slots, slots=slots, dtype="bf16")
    dec.load(weights)
    pre = pkg.Prefill(dec, max_rows=8192)
    server = pkg.Server(dec, pre)
    stream = stream_ctx(ctx)

    def run(read):
        st = serving.ContinuousStream(cfg.hidden, slots=slots)
        drv = serving.Driver(server, st.pool, slots)
        first = st.initial()
        drv.admit(first)
        server.sync()
        d0, p0 = drv.decoded, drv.prefilled
        started = {r.id for r in first}
        finished = []
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record(stream)
        for _ in range(steps):
            done = drv.step(read=read, keep=set() if not read else None)
            finished += done
            if done:
                new = [st.replacement() for _ in done]
                drv.admit(new)
                started |= {r.id for r in new}
        e1.record(stream)
        e1.synchronize()
        server.sync()
        wall = time.perf_counter() - t0
        return drv, e0.elapsed_time(e1), wall, drv.decoded - d0, drv.prefilled - p0, finished, st

    def clear(drv):
        for s in list(drv.owner):
            server.finish(s)
        drv.owner.clear()
        drv.left.clear()

    drv, ms, _, decoded, prefilled, finished, _ = run(False)
    clear(drv)
    # e2e: every step's outputs to the host; outputs kept for the invariance check.
    st = serving.ContinuousStream(cfg.hidden, slots=slots)
    drv2 = serving.Driver(server, st.pool, slots)
    first = st.initial()
    drv2.admit(first)
    server.sync()
    ids_full = []
    t0 = time.perf_counter()
    d0 = drv2.decoded
    for _ in range(steps):
        done = drv2.step(read=True, keep=None)
        if done:
            ids_full += done  # admitted before or inside the run: every step of it was read
            drv2.admit([st.replacement() for _ in done])
    wall = time.perf_counter() - t0
    e2e_tokens = drv2.decoded - d0
    clear(drv2)
    rng = np.random.default_rng(7)
    sample = [ids_full[i] for i in sorted(rng.choice(len(ids_full), min(check, len(ids_full)), replace=False))]
    same = 0
    for r in sample:
        alone = serving.Driver(server, st.pool, slots)
        alone.admit([r])
        keep = {r.id}
        for _ in range(r.steps):
            alone.step(read=True, keep=keep)
        same += int(all(np.array_equal(a, b) for a, b in zip(alone.outputs[r.id], drv2.outputs[r.id]))
                    and len(alone.outputs[r.id]) == r.steps == len(drv2.outputs[r.id]))
        clear(alone)
    out = {"slots": slots, "steps": steps, "decode_tokens": decoded, "prefill_rows": prefilled,
           "ms": round(ms, 3), "tokens_per_s": round(decoded / (ms / 1e3), 1),
           "mean_rows_per_step": round(decoded / steps, 2),
           "e2e_tokens_per_s": round(e2e_tokens / wall, 1),
           "invariance": f"{same}/{len(sample)} requests re-run alone bit-identical at every step",
           "schedule": "contexts U[64,2048] seed 2, lifetimes U[32,512], refills of 128 positions, "
                       "prefills of refills inside the timed region"}
    server.close()
    pre.close()
    dec.close()
    return out


def cpu_baseline(syn, shape, weights, seconds=10.0, max_steps=64):
    """The CPU oracle on this host's cores: decode steps at batch 1 from position 512 over a KV
    cache filled with N(0,1) values (a step's cost does not depend on the cache's values)."""
    import oracle

    threads = os.cpu_count() or 1
    stack = oracle.OracleStack(shape, syn.as_f32(weights), threads=threads)
    rng = np.random.default_rng(9)
    for l in range(shape.layers):
        stack.k_cache[l][:] = rng.standard_normal(stack.k_cache[l].shape, dtype=np.float32)
        stack.v_cache[l][:] = rng.standard_normal(stack.v_cache[l].shape, dtype=np.float32)
    x = rng.standard_normal((1, shape.hidden), dtype=np.float32)
    stack.decode_step([(PREFILL, 0)], x)
    t0 = time.perf_counter()
    n = 0
    while n < max_steps and time.perf_counter() - t0 < seconds:
        x = stack.decode_step([(PREFILL + 1 + n, 0)], x)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode steps at batch 1 from position {PREFILL + 1} (f32 oracle, "
                      f"{shape.layers} layers), {dt:.1f} s"}


def run_reference(args, rank, world, local):
    if rank != 0:
        return None
    import __graft_entry__ as entry

    entry.load_package()
    from tgtts_v4_b200 import synthetic as syn

    import oracle

    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=CAPACITY)
    weights = syn.make_weights(cfg, seed=0)
    threads = os.cpu_count() or 1
    stack = oracle.OracleStack(shape, weights, threads=threads)
    rng = np.random.default_rng(9)
    for l in range(shape.layers):
        stack.k_cache[l][:] = rng.standard_normal(stack.k_cache[l].shape, dtype=np.float32)
        stack.v_cache[l][:] = rng.standard_normal(stack.v_cache[l].shape, dtype=np.float32)
    x = rng.standard_normal((1, shape.hidden), dtype=np.float32)
    for i in range(args.warmup):
        x = stack.decode_step([(PREFILL + (i % 256), 0)], x)
    t0 = time.perf_counter()
    for i in range(args.steps):
        x = stack.decode_step([(PREFILL + ((args.warmup + i) % 256), 0)], x)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    sample = (f"{args.steps} decode steps at batch 1 from position {PREFILL} over a 512-position "
              f"cache, f32, all {threads} host threads")
    return {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config 2: 0.5B-shaped backbone decode at batch 1 from position 512",
                       "parallelism": "CPU, rank 0"},
            "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "tgtts-v4 cannot run here (Rust toolchain absent; GPU path is Vulkan): "
                    "the reference arm is the C restatement of its CPU f32 model (oracle/)"}


SERVE_METRIC = "serving decode tokens/s, all GPUs (0.5B-shaped bf16 backbone, <= 128 requests per GPU)"


def serve_config5(pkg, syn, ctx, torch, rank, world, local, requests, weights, clocks=None):
    """Config 5 on this rank's GPU: `requests` requests (prompts uniform 64-1024, decodes uniform
    64-768, seed 3, Poisson arrivals at 4096 a second, which keeps every GPU's 128 slots full),
    spread over the GPUs by a least-loaded rule every rank computes alike; each rank serves its share
    with one weight replica, continuous batching and no collective on the data path. Time: CUDA
    events on the rank's stream from the first admission to the last step (prefills included), max
    over ranks; per-step decode latency from events around each step, p50/p99 over all steps (max
    over ranks); each rank's busy time. Every rank returns the same dict."""
    from tgtts_v4_b200 import serving

    cfg = syn.S05B
    slots = 128
    shape = syn.shape_of(cfg, capacity=1024 + 768)
    dec = pkg.Decoder(ctx, shape, rows=slots, slots=slots, dtype="bf16")
    dec.load(weights)
    pre = pkg.Prefill(dec, max_rows=8192)
    server = pkg.Server(dec, pre)
    stream = stream_ctx(ctx)
    reqs, pool = serving.poisson_requests(requests, cfg.hidden, seed=3)
    mine = serving.assign_least_loaded(reqs, world)[rank]
    drv = serving.Driver(server, pool, slots)
    barrier(world)
    torch.cuda.synchronize()
    if clocks:
        clocks.__enter__()
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    e0 = ev()
    e0.record(stream)
    t0 = time.perf_counter()
    waiting = list(mine)
    marks = []
    while waiting or drv.owner:
        now = time.perf_counter() - t0
        free = len(drv.free_slots())
        ready = []
        while waiting and free and waiting[0].arrival <= now:
            ready.append(waiting.pop(0))
            free -= 1
        drv.admit(ready)
        if not drv.owner:
            time.sleep(max(0.0, min(0.001, waiting[0].arrival - now)))
            continue
        a, b = ev(), ev()
        a.record(stream)
        drv.step(read=False)
        b.record(stream)
        marks.append((a, b))
    e1 = ev()
    e1.record(stream)
    e1.synchronize()
    if clocks:
        clocks.__exit__(None, None, None)
    ms = e0.elapsed_time(e1)
    step_ms = sorted(x.elapsed_time(y) for x, y in marks)
    busy = [ms]
    decoded, prefilled, n_steps = drv.decoded, drv.prefilled, len(marks)
    p50, p99 = step_ms[len(step_ms) // 2], step_ms[int(len(step_ms) * 0.99)]
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([decoded, prefilled, n_steps], dtype=torch.float64)
        dist.all_reduce(t)
        decoded, prefilled, n_steps = (int(v) for v in t.tolist())
        lat = torch.tensor([p50, p99], dtype=torch.float64)
        dist.all_reduce(lat, op=dist.ReduceOp.MAX)
        p50, p99 = lat.tolist()
        per = torch.zeros(world, dtype=torch.float64)
        per[rank] = ms
        dist.all_reduce(per)
        busy = per.tolist()
    ms_max = max(busy)
    launches = n_steps * (len(dec.labels()) + 2)  # a step's kernels, the gather and the scatter
    server.close()
    pre.close()
    dec.close()
    return {"tokens_per_s": round(decoded / (ms_max / 1e3), 1), "decode_tokens": decoded,
            "prefill_tokens": prefilled, "steps": n_steps, "seconds": round(ms_max / 1e3, 3),
            "step_latency_ms": {"p50": round(p50, 4), "p99": round(p99, 4), "max_over_ranks": world > 1},
            "busy_s_per_rank": [round(v / 1e3, 3) for v in busy], "gpu_launches": launches,
            "requests": requests, "slots_per_gpu": slots,
            "how": "least-loaded split by prompt + decode positions; device time max over ranks"}


def run_serve(args, rank, world, local):
    """Config 5's own line (serve_config5): aggregate decode tokens/s over all GPUs."""
    import torch

    import __graft_entry__ as entry

    pkg = entry.load_package()
    from tgtts_v4_b200 import synthetic as syn

    torch.cuda.set_device(local)
    ctx = pkg.Context(local)
    weights = syn.make_weights(syn.S05B, seed=0, as_bits=True)
    clocks = Clocks(local)
    r = serve_config5(pkg, syn, ctx, torch, rank, world, local, args.requests, weights, clocks)
    result = None
    if rank == 0:
        c = clocks.summary()
        n_steps = r["steps"]
        result = {
            "metric": SERVE_METRIC, "value": r["tokens_per_s"], "unit": "tokens/s",
            "n_gpus": world, "steps": n_steps, "warmup": 0,
            "ms_per_step": round(r["seconds"] * 1e3 / max(1, n_steps // world), 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: N(0,0.02) weights seed 0, N(0,1) bf16-valued prompt rows, request lengths seed 3",
            "config": {"workload": "config 5: request-sharded serving, one weight replica per GPU, no collective",
                       "requests": args.requests, "slots_per_gpu": r["slots_per_gpu"], "prompt": "U[64,1024]",
                       "decode": "U[64,768]", "arrivals": "Poisson 4096/s (saturating)",
                       "parallelism": f"replicas x{world}, least-loaded assignment"},
            "prefill_tokens": r["prefill_tokens"], "decode_tokens": r["decode_tokens"], "seconds": r["seconds"],
            "step_latency_ms": r["step_latency_ms"], "busy_s_per_rank": r["busy_s_per_rank"],
            "gpu_launches": r["gpu_launches"],
            "clocks": {"sm_mhz": c["sm_mhz"], "sm_max_mhz": c["sm_max_mhz"], "reasons": c["reasons"]},
        }
    ctx.close()
    return result


def run_sweep(args, rank, world, local):
    """Decode step time by batch rows (`--sweep-rows`, default 1, 16, 64, 128): one decoder per size (rows = slots,
    capacity 2560, positions uniform 64-2048), `--steps` device-resident steps timed with CUDA
    events on the runtime's stream after `--warmup`; the projections' family as the decoder picks
    it (GEMVs below 16 rows, tcgen05 from 16)."""
    if rank != 0:
        return None
    import torch

    import __graft_entry__ as entry

    pkg = entry.load_package()
    from tgtts_v4_b200 import synthetic as syn

    torch.cuda.set_device(local)
    ctx = pkg.Context(local)
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=2560)
    weights = syn.make_weights(cfg, seed=0, as_bits=True)
    stream = stream_ctx(ctx)
    out = {}
    for rows in (int(v) for v in args.sweep_rows.split(",")):
        dec = pkg.Decoder(ctx, shape, rows=rows, slots=rows, dtype="bf16")
        dec.load(weights)
        pos = np.random.default_rng(2).integers(64, 2049, rows)
        words = [int(v) for v in pos] + (list(range(rows)) if rows > 1 else [])
        x = torch.randn(rows, cfg.hidden, device=f"cuda:{local}")
        y = torch.empty_like(x)
        for _ in range(args.warmup):
            dec.step_device(words, x.data_ptr(), y.data_ptr())
        ctx.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            dec.step_device(words, x.data_ptr(), y.data_ptr())
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        kv = sum(kv_bytes(shape, int(p)) for p in pos)
        out[str(rows)] = {"ms": round(ms, 4), "tokens_per_s": round(rows / ms * 1e3, 1),
                          "projections": ("tcgen05 split-K" if dec.split_k else "tcgen05 GEMM") if dec.tensor
                          else "gemv",
                          "hbm_gbs": round((shape.weight_bytes(2) + kv) / (ms * 1e6), 1)}
        dec.close()
    ctx.close()
    return {"workload": "decode step time by batch rows (0.5B-shaped bf16, positions U[64,2048])",
            "steps": args.steps, "warmup": args.warmup, "by_rows": out}


def run_gemm(args, rank, world, local):
    """Config 4's projection GEMMs, each alone: C = A B^T with A [rows][K] bf16 activations and B
    the layer's [N][K] bf16 weights (q/k/v 1280 x 1024, o 1024 x 1024, gate/up 8192 x 1024 with
    the SiLU epilogue, down 1024 x 4096), `--steps` launches in one program after `--warmup`,
    CUDA events at its ends; operands larger than L2 at the default 32768 rows."""
    if rank != 0:
        return None
    import torch

    import __graft_entry__ as entry

    pkg = entry.load_package()
    from tgtts_v4_b200 import synthetic as syn

    torch.cuda.set_device(local)
    ctx = pkg.Context(local)
    _, tc, peak_kind = peaks()
    shape = syn.shape_of(syn.S05B, capacity=64)
    M = args.rows
    out = {}
    for name, kernel, N, K in (("qkv_proj", "gemm", 1280, 1024), ("o_proj", "gemm", 1024, 1024),
                               ("gate_up_proj", "gemm_silu", 8192, 1024), ("down_proj", "gemm", 1024, 4096)):
        a, b = pkg.Memory(ctx, M * K * 2), pkg.Memory(ctx, N * K * 2)
        a.fill(0x3F803F80)  # bf16 1.0 pairs: finite operands, the values do not change the time
        b.fill(0x3F803F80)
        cb = M * N * 4 if kernel == "gemm" else M * (N // 2) * 2
        c = pkg.Memory(ctx, cb)
        p = pkg.params(shape, "bf16", rows=M, m=M, n=N, k=K)
        warm = pkg.Program(ctx, [(kernel, p, [(a, 0, a.nbytes), (b, 0, b.nbytes), (c, 0, cb)], name)] * max(1, args.warmup))
        warm.run()
        prog = pkg.Program(ctx, [(kernel, p, [(a, 0, a.nbytes), (b, 0, b.nbytes), (c, 0, cb)], name)] * args.steps)
        prog.run()
        ns = prog.elapsed_ns() / args.steps
        tflops = 2.0 * M * N * K / ns / 1e3
        out[name] = {"m": M, "n": N, "k": K, "us": round(ns / 1e3, 2), "tflops": round(tflops, 1),
                     "frac": round(tflops / tc, 4)}
        warm.close()
        prog.close()
        del a, b, c
    ctx.close()
    return {"workload": "config 4 projection GEMMs alone (tcgen05, persistent)", "steps": args.steps,
            "warmup": args.warmup, "peak_tflops": tc, "peak_source": peak_kind, "by_projection": out}


def run_local(args, rank, world, local):
    """VoxCPM2's local stacks (crates/graph/src/local): the patch sampler (10 Euler steps: 9 runs of
    the local DiT over each row's two sequences of 11 tokens) at 1 and 16 rows, and the local
    encoder at 16 rows, on VoxCPM2's widths (1024 wide, 4096 inner, 16 heads of 128 over 2 KV heads,
    patches of 4 frames of 64 channels) with 8 layers a stack (the checkpoint's layer count is not
    here), synthetic weights. One step is one sample of every row; `value` is patches/s at 16 rows
    with the inputs resident in HBM, `e2e` the same through tg_sampler_sample with host buffers."""
    if rank != 0:
        return None
    import torch

    import __graft_entry__ as entry
    import oracle

    pkg = entry.load_package()
    from tgtts_v4_b200 import local as loc
    from tgtts_v4_b200 import synthetic as syn

    torch.cuda.set_device(local)
    ctx = pkg.Context(local)
    stream = stream_ctx(ctx)
    hbm, _, peak_kind = peaks()
    cfg, timesteps = syn.LOCAL_VOXCPM2, 10
    shape = syn.local_shape(cfg)
    w = syn.make_sampler_weights(cfg, seed=0)
    steps, warm = max(1, args.steps // 10), max(3, args.warmup // 5)
    lines = {}
    for rows in (1, 16):
        s = loc.Sampler(ctx, shape, cfg.feat_dim, cfg.patch_size, timesteps, rows)
        s.load(w)
        mu, cond, noise, sampling = syn.make_sampler_inputs(cfg, rows, seed=1)
        dev = [torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{local}") for a in (mu.view(np.int16), cond, noise, sampling)]
        out = torch.empty_like(dev[1])
        ptrs = [t.data_ptr() for t in dev] + [out.data_ptr()]
        for _ in range(warm):
            s.sample_device(*ptrs)
        s.wait()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as clk:
            e0.record(stream)
            for _ in range(steps):
                s.sample_device(*ptrs)
            e1.record(stream)
            e1.synchronize()
        ms = e0.elapsed_time(e1) / steps
        for _ in range(warm):
            s.sample(mu, cond, noise, sampling)
        t0 = time.perf_counter()
        for _ in range(steps):
            s.sample(mu, cond, noise, sampling)
        e2e_ms = (time.perf_counter() - t0) * 1e3 / steps
        runs = len(s.steps())
        wb = s.weight_bytes
        lines[rows] = {"ms_per_sample": round(ms, 4), "patches_per_s": round(rows / ms * 1e3, 1),
                       "e2e_ms": round(e2e_ms, 4), "e2e_patches_per_s": round(rows / e2e_ms * 1e3, 1),
                       "dit_runs": runs, "weight_bytes_per_run": wb,
                       "weight_gbs": round(runs * wb / (ms / 1e3) / 1e9, 1),
                       "hbm_frac": round(runs * wb / (ms / 1e3) / 1e9 / hbm, 4),
                       "launches": len(s.labels()), "clocks": clk.summary()}
        s.close()
    e = loc.Encoder(ctx, shape, cfg.feat_dim, cfg.patch_size, 16)
    e.load(syn.make_encoder_weights(cfg, seed=0))
    patches = np.random.default_rng(3).standard_normal((16, cfg.feat_dim, cfg.patch_size)).astype(np.float32)
    for _ in range(warm):
        e.encode(patches)
    t = []
    for _ in range(steps):
        e.encode(patches)
        t.append(e.elapsed_ns() / 1e6)
    enc = {"rows": 16, "ms": round(statistics.median(t), 4), "weight_bytes": e.weight_bytes}
    e.close()
    # The CPU baseline: the oracle's sampler for one row on all host cores, one sample.
    cores = os.cpu_count() or 1
    ref = oracle.OracleLocal(shape, w, "feat_decoder.estimator.", 3 + 2 * cfg.patch_size, threads=cores)
    mu, cond, noise, sampling = syn.make_sampler_inputs(cfg, 1, seed=1)
    t0 = time.perf_counter()
    ref.sample(mu, cond, noise, sampling, timesteps, cfg.feat_dim, cfg.patch_size)
    cpu_ms = (time.perf_counter() - t0) * 1e3
    ctx.close()
    head = lines[16]
    return {"metric": "local sampler patches/s (VoxCPM2-wide local DiT, 10 Euler steps, 16 rows)",
            "value": head["patches_per_s"], "unit": "patches/s", "n_gpus": 1, "steps": steps, "warmup": warm,
            "ms_per_step": head["ms_per_sample"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic (seeded N(0, 0.02) weights; inputs as the reference's local tests)",
            "config": {"workload": "local sampler + encoder", "hidden": cfg.hidden, "inner": cfg.inner,
                       "heads": cfg.heads, "kv_heads": cfg.kv_heads, "head_dim": cfg.head_dim,
                       "layers": cfg.layers, "feat_dim": cfg.feat_dim, "patch_size": cfg.patch_size,
                       "timesteps": timesteps, "l2": "weights 277 MB a run > L2, no flush"},
            "e2e": {"value": head["e2e_patches_per_s"], "unit": "patches/s",
                    "h2d_bytes_per_step": 16 * (2 * cfg.hidden * 2 + 2 * cfg.feat_dim * cfg.patch_size * 4 + 8),
                    "d2h_bytes_per_step": 16 * cfg.feat_dim * cfg.patch_size * 4},
            "roofline": {"bound": "hbm", "achieved": head["weight_gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": head["hbm_frac"], "traffic": None, "peak_source": peak_kind},
            "cpu_baseline": {"value": round(1e3 / cpu_ms, 3), "unit": "patches/s", "cores": cores, "kind": "port",
                             "sample": "the oracle's sampler, 1 row, one sample of 10 steps"},
            "gpu_launches": head["launches"] * steps, "by_rows": lines, "encoder": enc}


def main():
    args = parse()
    rank, world, local = dist_init(args.gpus)
    if args.impl == "reference":
        res = run_reference(args, rank, world, local)
    elif args.workload == "serve":
        res = run_serve(args, rank, world, local)
    elif args.workload == "sweep":
        res = run_sweep(args, rank, world, local)
    elif args.workload == "gemm":
        res = run_gemm(args, rank, world, local)
    elif args.workload == "local":
        res = run_local(args, rank, world, local)
    else:
        res = run_ours(args, rank, world, local)
    if rank == 0 and res is not None:
        print(json.dumps(res))
        sys.stdout.flush()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
