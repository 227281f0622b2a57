"""Benchmark of the MoE FFN block (the ``moe_ffn_block`` hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl frank|reference]

One step = one ``moe_ffn_block`` call over one batch of synthetic tokens.
At N=1 the workload is the Mixtral-8x7B block (T=16384, H=4096, F=14336,
E=8, top-2, bf16, fp32 accumulation).  With N>1 (launched by torchrun, one
process per GPU, NCCL) every rank holds T tokens and E/N experts and the
block runs expert-parallel: tokens are dispatched to the ranks owning their
experts and the results combined back.  Scaling is strong: the global
batch stays T tokens, each rank holds T/N of them (the weak-scaling figure,
T tokens per rank, is reported under "weak").  The default N=1 run also
measures the decode blocks (T=1, T=8) and the fine-grained Zipf block under
"extra_configs".

Printed (rank 0, one JSON line):
  value       tokens/s over all ranks, inputs resident in HBM, device-timed with
              CUDA events, max over ranks
  e2e         the same through the public API with the step's x copied from
              pinned host memory and y copied back inside the timed region
  roofline    the dominant kernel (gate/up GEMM, or the fused decode kernel):
              algorithmic flops or bytes per launch / its CUDA-event duration
              (a separate loop of the same steps with events between the
              stages), against the measured peak (burst bf16 for a timed
              region under 2 s, HBM copy bandwidth for decode)
  cpu_baseline the CPU restatement of the reference (NumPy, grouped form) on a
              bounded token sample, rank 0 at N=1
--impl reference times that CPU restatement alone (the reference is a NumPy
oracle + IREE-compiled MLIR; IREE is not installable offline).
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

REPO = Path(__file__).resolve().parent
for _p in (REPO, REPO / "frank-models_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "moe_ffn_block tokens/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up GEMM launch
# (the CTA-pair kernel, tc2_grouped_gemm_kernel<0>).  Captured by ncu on the
# C3-shaped 2-expert case (626.7 MB read + 228.4 MB written,
# profiles/tc_grouped_gemm_c3_profile_2experts.md); C3 runs the same
# per-expert GEMM (4096 rows x 4096 x 2*14336) for 8 experts instead of 2, so
# its traffic is that capture x 4.
GATE_UP_TRAFFIC_BYTES = {"c3_mixtral_8x7b": 4 * (626.727e6 + 228.440e6)}
GATE_UP_TRAFFIC_SOURCE = {"c3_mixtral_8x7b": "ncu DRAM read + write of one gate/up launch on the C3-shaped "
                                             "2-expert case, x 4 (8 experts of the same GEMM shape)"}

# dram__bytes_read.sum + dram__bytes_write.sum of one decode_fused_kernel
# launch of the same workload (seed 0, 8 distinct experts), captured by ncu
# (76.670 MB read + 1.875 MB written, profiles/decode_fused_c5_T1.md).
DECODE_TRAFFIC_BYTES = {"c5_decode_T1": 76.670464e6 + 1.874688e6}


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling around the timed region.  The
    sampler is running (its first sample seen) before the region starts and
    keeps sampling ~250 ms after it ends, so even a millisecond-long region
    has samples on both sides of it."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = str(gpu_index)
        try:
            import torch

            self.idx = "GPU-" + str(torch.cuda.get_device_properties(gpu_index).uuid)
        except Exception:
            pass
        self.proc = None
        self.lines = []

    def _reader(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.lines.append(ln)

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._reader, daemon=True)
        self.thread.start()
        t0 = time.monotonic()
        while not self.lines and time.monotonic() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.thread.join(timeout=5)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in list(self.lines):
            f = [x.strip() for x in ln.split(",")]
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
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        if n and n[0]:
            return int(n[0])
    except Exception:
        pass
    return len(os.sched_getaffinity(0))


# ----------------------------------------------------------------- CPU arm --
def cpu_block_sample(cfg, x_f32, wr, w_up_p, w_gate_p, w_down_p, T_sample, reps=1):
    """Time the oracle's grouped restatement on the first T_sample tokens.
    Weights are packed [E, O, I] host arrays; the oracle reads them through
    [O, I, E] views (no copy).  Returns seconds per call."""
    from oracle import moe_oracle as O

    xs = x_f32[:T_sample]
    wu, wg, wd = (w.transpose(1, 2, 0) for w in (w_up_p, w_gate_p, w_down_p))
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        O.moe_ffn_block_grouped(xs, wr, wu, wg, wd, cfg.E, cfg.k, cfg.H, cfg.F, cfg.normalize)
        times.append(time.perf_counter() - t0)
    return min(times)


def host_weights_numpy(cfg, seed=0):
    import numpy as np

    rng = np.random.default_rng(seed)
    x = rng.standard_normal((max(cfg.T, 1), cfg.H), dtype=np.float32)
    wr = (rng.standard_normal((cfg.E, cfg.H), dtype=np.float32) * 0.02)
    wg = rng.standard_normal((cfg.E, cfg.F, cfg.H), dtype=np.float32)
    wg *= 0.02
    wu = rng.standard_normal((cfg.E, cfg.F, cfg.H), dtype=np.float32)
    wu *= 0.02
    wd = rng.standard_normal((cfg.E, cfg.H, cfg.F), dtype=np.float32)
    wd *= 0.02
    return x, wr, wu, wg, wd


def sample_tokens(cfg):
    return min(cfg.T, 256 if cfg.T >= 4096 else cfg.T)


def run_reference(args, cfg):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    x, wr, wu, wg, wd = host_weights_numpy(cfg)
    Ts = sample_tokens(cfg)
    for _ in range(args.warmup):
        cpu_block_sample(cfg, x, wr, wu, wg, wd, Ts)
    times = [cpu_block_sample(cfg, x, wr, wu, wg, wd, Ts) for _ in range(args.steps)]
    sec = sum(times) / len(times)
    v = Ts / sec
    cores = cpu_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(cfg, world),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{Ts} of {cfg.T} tokens per step, full H/F/E weights; the NumPy oracle's "
                                   f"grouped restatement (oracle/moe_oracle.py) on {cores} BLAS threads"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(cfg, world):
    return {"workload": cfg.name, "tokens_per_rank": cfg.T // world, "global_batch": cfg.T, "n_embd": cfg.H,
            "n_ff": cfg.F, "n_expert": cfg.E, "n_expert_used": cfg.k, "normalize_weights": cfg.normalize,
            "parallelism": f"ep{world}",
            "l2": "inputs larger than L2: expert weights and per-step activations exceed the 126 MB L2"}


# ----------------------------------------------------------------- GPU arm --
def _barrier(dist):
    import torch

    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(dist, dev, v: float) -> float:
    import torch

    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _gemm_peak(pk, timed_s):
    """The bf16 denominator: the burst figure for a kernel timed in a region
    shorter than ~2 s (the clocks stay near maximum), else the sustained one."""
    key = "bf16_tflops" if timed_s < 2.0 else "bf16_tflops_sustained"
    return float(pk[key]), key


def bench_block_1gpu(args, cfg, dev, local, cpu=True):
    """One configuration on one GPU.  Returns the measurement dict (value,
    ms_per_step, roofline, stage_ms, e2e, gpu_launches, clocks, cpu_baseline)."""
    import torch

    from frank_b200 import configs, ops

    wr, wu, wg, wd = configs.block_weights_packed_torch(cfg, dev, seed=0)
    block = ops.MoEFFNBlock(wr, ops.PackedExperts(wu), ops.PackedExperts(wg), ops.PackedExperts(wd), cfg.E,
                            cfg.k, cfg.normalize, dtype=torch.bfloat16, out_dtype=torch.float32)
    x = configs.block_x_torch(cfg, dev, seed=0)
    y = torch.empty((cfg.T, cfg.H), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    decode = cfg.T <= 64
    graphed = None
    if decode:
        # decode steps are launch-bound: replay the block from a CUDA graph
        l_cap = ops.launch_count()
        graphed = ops.GraphedMoEFFN(block, cfg.T, dev)
        graphed_launches = (ops.launch_count() - l_cap) // 2  # warm-up call + captured call
        graphed.x.copy_(x)

        def step():
            graphed.replay()
    else:
        def step():
            block(x, out=y)

    for _ in range(args.warmup):
        step()
    _barrier(None)

    # ---- value: inputs resident in HBM, no instrumentation in the loop ------
    # Decode-sized steps touch less than the 126 MB L2 (T=1 reads ~75 MB of
    # weights): flush L2 between steps (a 256 MiB write, outside the timed
    # spans) and time every step on its own.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if decode else None
    l0 = ops.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)] if decode else []
    with ClockSampler(local) as clk:
        _barrier(None)
        ev0.record(stream)
        for i in range(args.steps):
            if decode:
                flush.zero_()
                step_ev[i][0].record(stream)
            step()
            if decode:
                step_ev[i][1].record(stream)
        ev1.record(stream)
        _barrier(None)
    launches = graphed_launches * args.steps if decode else ops.launch_count() - l0
    region_ms = ev0.elapsed_time(ev1)
    ms = (sum(a.elapsed_time(b) for a, b in step_ev) if decode else region_ms) / args.steps

    # ---- per-stage device times: a separate loop of the same steps ---------
    n_prof = min(args.steps, 10)
    acc = {}
    if decode:
        # the timed graph carries no stage events; a second capture of the same
        # block records events between the stages (replayed with the same flush)
        ops.profile_stages(2)
        g2 = ops.GraphedMoEFFN(block, cfg.T, dev)
        ops.profile_stages(False)
        g2.x.copy_(x)
        for _ in range(n_prof):
            flush.zero_()
            g2.replay()
            for kk, vv in ops.profile_read().items():
                acc[kk] = acc.get(kk, 0.0) + vv / n_prof
        del g2
    else:
        ops.profile_stages(True)
        for _ in range(n_prof):
            block(x, out=y)
            for kk, vv in ops.profile_read().items():
                acc[kk] = acc.get(kk, 0.0) + vv / n_prof
        ops.profile_stages(False)
    stage_ms = acc
    _, _, rid = block(x, return_routing=True)
    rid_h = rid.cpu()
    n_distinct = int(torch.unique(rid_h).numel())
    rows = torch.bincount(rid_h.reshape(-1).long(), minlength=cfg.E)

    pk, pk_kind = peaks()
    res = {"value": cfg.T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
           "tflops": cfg.flops / (ms / 1e3) / 1e12, "config": config_dict(cfg, 1), "stage_ms": stage_ms,
           "gpu_launches": int(launches), "clocks": clk.summary()}
    if decode:
        res["config"]["l2"] = "L2 flushed (256 MiB write) before every timed step; steps timed individually"
        # weight streaming, HBM-bound.  Algorithmic bytes of the block =
        # distinct experts x 3 matrices x F x H bf16 + router + activations.
        blk_bytes = (n_distinct * 3 * cfg.F * cfg.H * 2 + cfg.E * cfg.H * 4 + cfg.T * cfg.H * 2 + cfg.T * cfg.H * 4)
        fused = cfg.k * cfg.T <= cfg.E
        # fused: the one cooperative launch sits between the first two stage
        # marks (the later marks follow it back to back, so their spans hold
        # no kernel, only the event resolution)
        k_ms = stage_ms["route"] if fused else stage_ms["gate_up_gemm"]
        k_bytes = blk_bytes if fused else (n_distinct * 2 * cfg.F * cfg.H * 2 + cfg.k * cfg.T * (cfg.H + cfg.F) * 2)
        achieved = k_bytes / (k_ms / 1e3) / 1e9
        peak = float(pk["hbm_gbs"])
        tr = DECODE_TRAFFIC_BYTES.get(cfg.name) if fused else None
        res["roofline"] = {
            "kernel": "decode_fused_kernel (whole block)" if fused else "tc_grouped_gemm<SWIGLU> (gate/up GEMM + swiglu)",
            "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": f"{pk_kind} hbm_gbs", "traffic": tr,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch, same workload"
                              if tr else None,
            "bytes_per_launch": k_bytes, "ms_per_launch": k_ms, "distinct_experts": n_distinct,
        }
        res["block_hbm_gbs"] = blk_bytes / (ms / 1e3) / 1e9
        res["block_frac_of_hbm"] = res["block_hbm_gbs"] / peak
    else:
        gu_flops = 4.0 * cfg.k * cfg.T * cfg.H * cfg.F
        gu_ms = stage_ms["gate_up_gemm"]
        achieved = gu_flops / (gu_ms / 1e3) / 1e12
        peak, peak_key = _gemm_peak(pk, region_ms / 1e3)
        tr = GATE_UP_TRAFFIC_BYTES.get(cfg.name)
        res["roofline"] = {
            "kernel": "tc_grouped_gemm<SWIGLU> (gate/up GEMM + swiglu)", "bound": "tensor",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{pk_kind} {peak_key} (timed region {region_ms / 1e3:.2f} s)",
            "frac_of_sustained": achieved / float(pk["bf16_tflops_sustained"]),
            "traffic": tr, "traffic_source": GATE_UP_TRAFFIC_SOURCE.get(cfg.name) if tr else None,
            "flops_per_launch": gu_flops, "ms_per_launch": gu_ms,
            "stage_ms_from": f"separate loop of {n_prof} steps with stage events",
        }
        res["block_frac_of_peak"] = res["tflops"] / peak
    if cfg.E >= 16:
        res["rows_per_expert"] = {"max": int(rows.max()), "mean": float(rows.float().mean()),
                                  "below_64": int((rows < 64).sum())}

    # ---- e2e: host x in, host y out, through the public API ---------------
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((cfg.T, cfg.H), dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)
    pipe = None
    host_graph = None
    if decode:
        # decode: copy in, block and copy out captured as one graph
        host_graph = ops.GraphedHostMoEFFN(block, cfg.T, dev)
        host_graph.x_host.copy_(x_host)
    if not decode and cfg.T >= 1024:
        pipe = ops.HostPipeline(block, cfg.T, cfg.H, x.dtype, torch.float32, depth=2, device=dev)

    def e2e_step(last):
        if host_graph is not None:
            # pinned host tokens -> device -> block -> pinned host result, one graph launch
            host_graph.replay()
        elif pipe is None:
            # one copy each way around the block
            x_dev.copy_(x_host, non_blocking=True)
            block(x_dev, out=y)
            y_host.copy_(y, non_blocking=True)
        else:
            # public host-buffer API: every step copies its tokens in and its
            # result out; the copies of neighbouring steps overlap this
            # step's block on separate streams; the last copy out is waited for
            done = pipe.submit(x_host, y_host)
            if last:
                stream.wait_event(done)

    for _ in range(min(args.warmup, 2)):
        e2e_step(True)
    _barrier(None)
    ev0.record(stream)
    for i in range(args.steps):
        e2e_step(i == args.steps - 1)
    ev1.record(stream)
    _barrier(None)
    e2e_ms = ev0.elapsed_time(ev1) / args.steps
    res["e2e"] = {"value": cfg.T / (e2e_ms / 1e3), "unit": "tokens/s",
                  "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                  "d2h_bytes_per_step": y_host.numel() * y_host.element_size()}
    del pipe
    if cpu:
        res["cpu_baseline"] = cpu_baseline_from_device(cfg, x, block)
    return res


def run_frank(args, cfg):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        return run_frank_ep(args, cfg, dev, rank, world, local)
    res = bench_block_1gpu(args, cfg, dev, local, cpu=not args.no_cpu_baseline)
    torch.cuda.empty_cache()
    line = {
        "metric": METRIC, "value": res.pop("value"), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": res.pop("ms_per_step"), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights; no dataset)",
    }
    line.update(res)
    if args.extras and cfg.name == configs_default():
        from frank_b200 import configs

        extra = {}
        for c in (configs.c5(1), configs.c5(8), configs.c5(32), configs.c5(64), configs.C4):
            r = bench_block_1gpu(args, c, dev, local, cpu=not args.no_cpu_baseline)
            torch.cuda.empty_cache()
            extra[c.name] = r
        extra[configs.C2.name] = bench_mul_mat_id(args, configs.C2)
        torch.cuda.empty_cache()
        line["extra_configs"] = extra
    print(json.dumps(line), flush=True)


def configs_default():
    return "c3_mixtral_8x7b"


def run_frank_ep(args, cfg, dev, rank, world, local):
    """Expert parallelism over ``world`` GPUs: strong scaling at the
    configuration's global token count (each rank holds T / world of the
    same seeded tokens) for ``value``; the weak-scaling figure (T tokens per
    rank) rides along under ``weak``."""
    import torch
    import torch.distributed as dist

    from frank_b200 import configs, ep, ops

    dist.init_process_group("nccl", device_id=dev)
    runner = ep.ExpertParallelMoE.synthetic(cfg, rank, world, dev, seed=0)
    stream = torch.cuda.current_stream()

    def measure(cfg, T_rank, x, e2e=True):
        y = torch.empty((T_rank, cfg.H), dtype=torch.float32, device=dev)
        for _ in range(args.warmup):
            runner(x, out=y)
        _barrier(dist)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0 = ops.launch_count()
        with ClockSampler(local) as clk:
            _barrier(dist)
            ev0.record(stream)
            for _ in range(args.steps):
                runner(x, out=y)
            ev1.record(stream)
            _barrier(dist)
        launches = ops.launch_count() - l0
        ms = _max_over_ranks(dist, dev, ev0.elapsed_time(ev1)) / args.steps
        # phases and rows received: a separate profiled loop
        runner.profile = True
        for _ in range(min(args.steps, 5)):
            runner(x, out=y)
        runner.profile = False
        mine = {"rank": rank, "phase_ms": runner.phase_ms(), "rows_received": runner.rows_received(),
                "mode": runner.mode}
        info = [None] * world
        dist.all_gather_object(info, mine)
        out = {"value": cfg.T * (world if T_rank == cfg.T else 1) / (ms / 1e3), "ms_per_step": ms,
               "tokens_per_rank": T_rank, "gpu_launches": int(launches), "clocks": clk.summary(),
               "ep_ranks": info}
        r = [i["rows_received"] for i in info]
        out["rows_per_rank"] = {"max": max(r), "mean": sum(r) / len(r), "max_over_mean": max(r) / (sum(r) / len(r))}
        if e2e:
            x_host = x.cpu().pin_memory()
            y_host = torch.empty((T_rank, cfg.H), dtype=torch.float32).pin_memory()
            del y
            torch.cuda.empty_cache()
            pipe = ops.HostPipeline(runner, T_rank, cfg.H, x.dtype, torch.float32, depth=2, device=dev)
            for _ in range(2):
                stream.wait_event(pipe.submit(x_host, y_host))
            _barrier(dist)
            ev0.record(stream)
            for i in range(args.steps):
                done = pipe.submit(x_host, y_host)
                if i == args.steps - 1:
                    stream.wait_event(done)
            ev1.record(stream)
            _barrier(dist)
            e2e_ms = _max_over_ranks(dist, dev, ev0.elapsed_time(ev1)) / args.steps
            tot = T_rank * world
            out["e2e"] = {"value": tot / (e2e_ms / 1e3), "unit": "tokens/s",
                          "h2d_bytes_per_step": x_host.numel() * x_host.element_size() * world,
                          "d2h_bytes_per_step": y_host.numel() * y_host.element_size() * world}
        return out

    # strong scaling: the global batch of cfg.T seeded tokens split over the ranks
    T_rank = cfg.T // world
    x_all = configs.block_x_torch(cfg, dev, seed=0)
    x = x_all[rank * T_rank:(rank + 1) * T_rank].contiguous()
    del x_all
    strong = measure(cfg, T_rank, x)
    # weak scaling: cfg.T tokens on every rank
    weak = measure(cfg, cfg.T, configs.block_x_torch(cfg, dev, seed=rank), e2e=False) if args.extras else None
    extra = None
    if args.extras and cfg.name == configs_default():
        # the fine-grained Zipf block, strong scaling: per-rank load under skew
        c4 = configs.C4
        runner = None
        torch.cuda.empty_cache()
        runner = ep.ExpertParallelMoE.synthetic(c4, rank, world, dev, seed=0)
        xa = configs.block_x_torch(c4, dev, seed=0)
        Tr = c4.T // world
        xr = xa[rank * Tr:(rank + 1) * Tr].contiguous()
        del xa
        extra = {c4.name: measure(c4, Tr, xr, e2e=False)}
        extra[c4.name]["placement"] = "contiguous expert ranges"
        # the same, with the experts placed by the load of a calibration
        # batch (other seeded tokens of the same distribution)
        xc = configs.block_x_torch(c4, dev, seed=1)[rank * Tr:(rank + 1) * Tr].contiguous()
        placement = ep.balanced_placement(ep.measure_expert_load(xc, runner.wr, c4.k, c4.normalize, c4.E), world)
        del xc
        runner = None
        torch.cuda.empty_cache()
        runner = ep.ExpertParallelMoE.synthetic(c4, rank, world, dev, seed=0, placement=placement)
        bal = measure(c4, Tr, xr, e2e=False)
        bal["placement"] = "load-balanced from a calibration batch (seed 1)"
        extra[c4.name + "_balanced"] = bal
    if rank == 0:
        line = {
            "metric": METRIC, "value": strong["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": strong["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights; no dataset)",
            "config": config_dict(cfg, world),
            "e2e": strong["e2e"], "gpu_launches": strong["gpu_launches"], "clocks": strong["clocks"],
            "ep_ranks": strong["ep_ranks"], "rows_per_rank": strong["rows_per_rank"],
            "tflops": cfg.flops / (strong["ms_per_step"] / 1e3) / 1e12,
        }
        if weak is not None:
            line["weak"] = {k: weak[k] for k in ("value", "ms_per_step", "tokens_per_rank", "rows_per_rank")}
        if extra:
            line["extra_configs"] = extra
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_mul_mat_id(args, cfg):
    """mul_mat_id alone (bf16 in, fp32 accumulate and output), one GPU."""
    print(json.dumps(bench_mul_mat_id(args, cfg)), flush=True)


def bench_mul_mat_id(args, cfg):
    """The mul_mat_id bench line (dict): grouped GEMM over expert-sorted
    columns, inputs resident on the device."""
    import numpy as np
    import torch

    from frank_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    w = torch.empty((cfg.E, cfg.n_out, cfg.n_in), dtype=torch.float32, device=dev).normal_(0, 0.02, generator=g)
    wp = ops.PackedExperts(w.bfloat16())
    del w
    x = torch.empty((cfg.n_in, 1, cfg.T), dtype=torch.float32, device=dev).normal_(0, 1, generator=g)
    inp = x.expand(cfg.n_in, cfg.k, cfg.T).contiguous().bfloat16()
    rng = np.random.default_rng(0)
    ids = torch.from_numpy(np.stack([rng.permutation(cfg.E)[: cfg.k] for _ in range(cfg.T)], axis=1)
                           .astype(np.int32)).to(dev)
    for _ in range(args.warmup):
        ops.mul_mat_id(wp, inp, ids, check_ids=False)
    torch.cuda.synchronize()
    l0 = ops.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        ev0.record()
        for _ in range(args.steps):
            ops.mul_mat_id(wp, inp, ids, check_ids=False)
        ev1.record()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / args.steps
    pk, pk_kind = peaks()
    tf = cfg.flops / (ms / 1e3) / 1e12
    gpk, gkey = _gemm_peak(pk, ms * args.steps / 1e3)
    line = {"metric": "mul_mat_id tokens/s", "value": cfg.T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg.name, "n_tokens": cfg.T, "n_in": cfg.n_in, "n_out": cfg.n_out,
                       "n_expert": cfg.E, "n_expert_used": cfg.k, "output": "fp32 [n_out, k, T]"},
            "tflops": tf, "frac_of_sustained_bf16": tf / float(pk["bf16_tflops_sustained"]),
            "roofline": {"kernel": "mul_mat_id (gather_cols + tc_grouped_gemm + scatter_out)", "bound": "tensor",
                         "achieved": tf, "peak": gpk, "unit": "TFLOP/s", "frac": tf / gpk,
                         "peak_source": f"{pk_kind} {gkey} (the whole call timed)", "traffic": None},
            "gpu_launches": int(ops.launch_count() - l0), "clocks": clk.summary()}
    return line


def cpu_baseline_from_device(cfg, x, block):
    """The oracle on the same weights (copied from the device) and the first
    sample tokens, on all host BLAS threads."""
    import numpy as np

    Ts = sample_tokens(cfg)
    xs = x[:Ts].float().cpu().numpy()
    wr = block.wr.float().cpu().numpy()
    wu, wg, wd = (t.float().cpu().numpy() for t in (block.w_up, block.w_gate, block.w_down))
    cpu_block_sample(cfg, xs, wr, wu, wg, wd, Ts)  # warm caches / thread pool
    sec = cpu_block_sample(cfg, xs, wr, wu, wg, wd, Ts, reps=2)
    cores = cpu_threads()
    return {"value": Ts / sec, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{Ts} of {cfg.T} tokens, same weights; NumPy grouped restatement of oracles/moe.py "
                      f"(oracle/moe_oracle.py), {cores} BLAS threads"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c3_mixtral_8x7b")
    ap.add_argument("--impl", default="frank", choices=["frank", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", dest="extras", action="store_false",
                    help="skip the extra configurations (decode T=1, T=8 and the fine-grained block)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)  # at least 3 untimed warm-up steps
    from frank_b200 import configs

    if args.config == configs.C2.name:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm covers moe_ffn_block configs"}))
            return
        run_mul_mat_id(args, configs.C2)
        return
    cfg = configs.BLOCK_CONFIGS[args.config]
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_frank(args, cfg)


if __name__ == "__main__":
    main()
