"""Benchmark of the MoE FFN block (the ``moe_ffn_block`` hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl frank|reference]

One step = one ``moe_ffn_block`` call over one batch of synthetic tokens.
At N=1 the workload is the Mixtral-8x7B block (T=16384, H=4096, F=14336,
E=8, top-2, bf16, fp32 accumulation).  With N>1 (launched by torchrun, one
process per GPU, NCCL) every rank holds T tokens and E/N experts and the
block runs expert-parallel: tokens are dispatched to the ranks owning their
experts and the results combined back (weak scaling: T tokens per rank).

Printed (rank 0, one JSON line):
  value       tokens/s over all ranks, inputs resident in HBM, device-timed with
              CUDA events, max over ranks
  e2e         the same through the public API with the step's x copied from
              pinned host memory and y copied back inside the timed region
  roofline    the gate/up GEMM (dominant kernel): algorithmic flops per launch /
              its CUDA-event duration inside the timed region, against the
              measured dense bf16 peak
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

# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up GEMM launch.
# Captured by ncu on the C3-shaped 2-expert case (558 MB read + 224 MB
# written, profiles/tc_grouped_gemm_c3_profile_2experts.md); C3 runs the same
# per-expert GEMM (4096 rows x 4096 x 2*14336) for 8 experts instead of 2, so
# its traffic is that capture x 4.
GATE_UP_TRAFFIC_BYTES = {"c3_mixtral_8x7b": 4 * (558.111e6 + 223.502e6)}

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
    """nvidia-smi clocks/throttle sampling during the timed region."""

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

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
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
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(cfg, world),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{Ts} of {cfg.T} tokens per step, full H/F/E weights; the NumPy oracle's "
                                   f"grouped restatement (oracle/moe_oracle.py) on {cores} BLAS threads"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(cfg, world):
    return {"workload": cfg.name, "tokens_per_rank": cfg.T, "global_batch": cfg.T * world, "n_embd": cfg.H,
            "n_ff": cfg.F, "n_expert": cfg.E, "n_expert_used": cfg.k, "normalize_weights": cfg.normalize,
            "parallelism": f"ep{world}",
            "l2": "inputs larger than L2: expert weights and per-step activations exceed the 126 MB L2"}


# ----------------------------------------------------------------- GPU arm --
def run_frank(args, cfg):
    import numpy as np
    import torch

    from frank_b200 import configs, ops

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    graphed = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
        from frank_b200 import ep

        runner = ep.ExpertParallelMoE.synthetic(cfg, rank, world, dev, seed=0)
        block_call = runner.__call__
    else:
        runner = None
        dist = None
        wr, wu, wg, wd = configs.block_weights_packed_torch(cfg, dev, seed=0)
        block = ops.MoEFFNBlock(wr, ops.PackedExperts(wu), ops.PackedExperts(wg), ops.PackedExperts(wd), cfg.E,
                                cfg.k, cfg.normalize, dtype=torch.bfloat16, out_dtype=torch.float32)
        block_call = block.__call__
        graphed = None
        if cfg.T <= 64:
            # decode steps are launch-bound: replay the block from a CUDA graph
            l_cap = ops.launch_count()
            graphed = ops.GraphedMoEFFN(block, cfg.T, dev)
            graphed_launches = (ops.launch_count() - l_cap) // 2  # warm-up call + captured call
            block_call = graphed.__call__
    x = configs.block_x_torch(cfg, dev, seed=rank)
    y = torch.empty((cfg.T, cfg.H), dtype=torch.float32, device=dev)
    e2e_call = block_call
    if graphed is not None:
        graphed.x.copy_(x)  # the resident input of the timed replays

        def block_call(x_, out=None):  # noqa: F811 -- value loop: replay only, x already resident
            return graphed.replay()
    stream = torch.cuda.current_stream()

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        block_call(x, out=y)
    barrier()

    # ---- value: inputs resident in HBM -------------------------------------
    ops.profile_stages(True)
    if runner is not None:
        runner.profile = True
    # Decode-sized steps touch less than the 126 MB L2 (T=1 reads ~75 MB of
    # weights): flush L2 between steps (a 256 MiB write, outside the timed
    # spans) and time every step on its own.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if cfg.T <= 64 else None
    l0 = ops.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)] if flush is not None else []
    with ClockSampler(local) as clk:
        barrier()
        ev0.record(stream)
        for i in range(args.steps):
            if flush is not None:
                flush.zero_()
                step_ev[i][0].record(stream)
            block_call(x, out=y)
            if flush is not None:
                step_ev[i][1].record(stream)
        ev1.record(stream)
        barrier()
    launches = ops.launch_count() - l0
    ops.profile_stages(False)
    if world == 1 and graphed is not None:
        # The timed graph carries no stage events; a second capture of the same
        # block with events between the stages gives the per-stage device times
        # (replayed with the same L2 flush, averaged).
        launches = graphed_launches * args.steps
        ops.profile_stages(2)
        g2 = ops.GraphedMoEFFN(block, cfg.T, dev)
        ops.profile_stages(False)
        acc = {}
        for _ in range(args.steps):
            flush.zero_()
            g2.x.copy_(x)
            g2.replay()
            for kk, vv in ops.profile_read().items():
                acc[kk] = acc.get(kk, 0.0) + vv / args.steps
        stage_ms = acc
        del g2
    else:
        stage_ms = ops.profile_read() if world == 1 else {}
    ep_info = None
    if runner is not None:
        runner.profile = False
        mine = {"rank": rank, "phase_ms": runner.phase_ms(), "rows_received": runner.rows_received(), "mode": runner.mode}
        ep_info = [None] * world
        dist.all_gather_object(ep_info, mine)
    if flush is not None:
        ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in step_ev)) / args.steps
    else:
        ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    value = cfg.T * world / (ms / 1e3)
    n_distinct = None
    if world == 1:
        _, _, rid = block(x, return_routing=True)
        n_distinct = int(torch.unique(rid).numel())

    # ---- e2e: host x in, host y out, through the public API ---------------
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((cfg.T, cfg.H), dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)
    pipe = None
    if graphed is None and cfg.T >= 1024:
        del y
        torch.cuda.empty_cache()
        pipe = ops.HostPipeline(e2e_call, cfg.T, cfg.H, x.dtype, torch.float32, depth=2, device=dev)

    def e2e_step(last):
        if graphed is not None or cfg.T < 1024:
            # decode: one copy each way around the (graph-replayed) block
            x_dev.copy_(x_host, non_blocking=True)
            e2e_call(x_dev, out=y)
            y_host.copy_(y, non_blocking=True)
        else:
            # public host-buffer API: every step copies its tokens in and its
            # result out; the copies of neighbouring steps overlap this
            # step's block on separate streams; the last copy out is waited for
            done = pipe.submit(x_host, y_host)
            if last:
                stream.wait_event(done)

    for i in range(min(args.warmup, 2)):
        e2e_step(True)
    barrier()
    ev0.record(stream)
    for i in range(args.steps):
        e2e_step(i == args.steps - 1)
    ev1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    e2e = {"value": cfg.T * world / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": x_host.numel() * x_host.element_size() * world,
           "d2h_bytes_per_step": y_host.numel() * y_host.element_size() * world}

    if rank != 0:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    pk, pk_kind = peaks()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights; no dataset)",
        "config": config_dict(cfg, world),
        "tflops": cfg.flops * world / (ms / 1e3) / 1e12,
    }
    if flush is not None:
        line["config"]["l2"] = "L2 flushed (256 MiB write) before every timed step; steps timed individually"
    if stage_ms and cfg.T <= 64:
        # decode: weight streaming, HBM-bound.  Algorithmic bytes of the block =
        # distinct experts x 3 matrices x F x H bf16 + router + activations.
        # Small decode blocks run as one fused kernel, so the roofline kernel
        # is the whole block (the sum of the recorded stages).
        blk_bytes = (n_distinct * 3 * cfg.F * cfg.H * 2 + cfg.E * cfg.H * 4 + cfg.T * cfg.H * 2 + cfg.T * cfg.H * 4)
        fused = cfg.k * cfg.T <= cfg.E
        # fused: the one cooperative launch sits between the first two stage
        # marks (the later marks follow it back to back, so their spans hold
        # no kernel, only the event resolution)
        k_ms = stage_ms["route"] if fused else stage_ms["gate_up_gemm"]
        k_bytes = blk_bytes if fused else (n_distinct * 2 * cfg.F * cfg.H * 2 + cfg.k * cfg.T * (cfg.H + cfg.F) * 2)
        achieved = k_bytes / (k_ms / 1e3) / 1e9
        peak = float(pk["hbm_gbs"])
        line["roofline"] = {
            "kernel": "decode_fused_kernel (whole block)" if fused else "tc_grouped_gemm<SWIGLU> (gate/up GEMM + swiglu)",
            "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_source": f"{pk_kind} hbm_gbs",
            "traffic": DECODE_TRAFFIC_BYTES.get(cfg.name) if fused else None,
            "bytes_per_launch": k_bytes, "ms_per_launch": k_ms,
            "distinct_experts": n_distinct,
        }
        line["stage_ms"] = stage_ms
        line["block_hbm_gbs"] = blk_bytes / (ms / 1e3) / 1e9
        line["block_frac_of_hbm"] = line["block_hbm_gbs"] / peak
    elif stage_ms:
        gu_flops = 4.0 * cfg.k * cfg.T * cfg.H * cfg.F
        gu_ms = stage_ms["gate_up_gemm"]
        achieved = gu_flops / (gu_ms / 1e3) / 1e12
        peak = float(pk["bf16_tflops_sustained"])
        line["roofline"] = {
            "kernel": "tc_grouped_gemm<SWIGLU> (gate/up GEMM + swiglu)", "bound": "tensor",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{pk_kind} bf16_tflops_sustained", "traffic": GATE_UP_TRAFFIC_BYTES.get(cfg.name),
            "flops_per_launch": gu_flops, "ms_per_launch": gu_ms,
        }
        line["stage_ms"] = stage_ms
        line["block_frac_of_peak"] = line["tflops"] / peak
    if ep_info:
        line["ep_ranks"] = ep_info
    line["e2e"] = e2e
    line["gpu_launches"] = int(launches)
    line["clocks"] = clk.summary()
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_from_device(cfg, x, block if world == 1 else None)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_mul_mat_id(args, cfg):
    """mul_mat_id alone (bf16 in, fp32 accumulate and output), one GPU."""
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
    line = {"metric": "mul_mat_id tokens/s", "value": cfg.T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg.name, "n_tokens": cfg.T, "n_in": cfg.n_in, "n_out": cfg.n_out,
                       "n_expert": cfg.E, "n_expert_used": cfg.k, "output": "fp32 [n_out, k, T]"},
            "tflops": tf, "frac_of_sustained_bf16": tf / float(pk["bf16_tflops_sustained"]),
            "gpu_launches": int(ops.launch_count() - l0), "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


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
