"""bf16 tensor-core (tcgen05) path vs the oracle.

Reference values are the oracle evaluated in float64 on the same
bf16-rounded inputs.  Tolerance: max-abs <= 2e-2 x output RMS for the block
(bf16 h and y), tighter for mul_mat_id (fp32 output, only the accumulation
order differs).  Routing is held to the strict tier (tests/utils.py
``strict_routing``): the GPU's expert ids equal the oracle's top-k on float64
logits for every token whose k-th/(k+1)-th logit gap exceeds the fp32
accumulation bound, and the oracle then runs with its OWN routing (the GPU's
ids only on near-tied tokens where they differ, with float64 weights).
"""

import numpy as np
import pytest
import torch

from frank_b200 import configs, ops
from oracle import moe_oracle as O
from tests.utils import rms_rel_maxabs, strict_route

pytestmark = pytest.mark.gpu

BLOCK_TOL = 2e-2
MMID_TOL = 1e-3


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().bfloat16()


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("O_,I,E,k,T,kind", [
    (512, 256, 8, 2, 300, "uniform"),
    (256, 128, 4, 1, 1, "uniform"),        # one token
    (144, 72, 6, 2, 129, "one"),           # ragged N (144 % 256 != 0), K % 64 != 0, all on one expert
    (256, 64, 16, 4, 200, "sparse"),       # empty experts
    (1024, 512, 8, 2, 1000, "uniform"),
    (208, 136, 8, 2, 260, "uniform"),      # tiled transposes with partial 64-wide tiles on every axis
])
def test_mul_mat_id_bf16(O_, I, E, k, T, kind):
    rng = np.random.default_rng(O_ + T)
    w = (rng.standard_normal((O_, I, E)) * 0.05).astype(np.float32)
    x = rng.standard_normal((I, k, T)).astype(np.float32)
    if kind == "uniform":
        ids = rng.integers(0, E, size=(k, T))
    elif kind == "one":
        ids = np.full((k, T), E // 2)
    else:
        ids = rng.choice([1, E - 1], size=(k, T))
    ids = ids.astype(np.int32)
    wb, xb = _bf16(w), _bf16(x)
    out = ops.mul_mat_id(wb, xb, torch.from_numpy(ids).cuda())
    ref = O.mul_mat_id_grouped(_f64(wb), _f64(xb), ids)
    assert rms_rel_maxabs(out.cpu().numpy(), ref) <= MMID_TOL
    assert ops.read_device_error() == 0


def _block_check(cfg, seed):
    x, wr, wu, wg, wd = configs.block_inputs_numpy(cfg, seed=seed)
    xb = _bf16(x)
    tb = [_bf16(w) for w in (wu, wg, wd)]
    block = ops.MoEFFNBlock(torch.from_numpy(wr).cuda(), *tb, cfg.E, cfg.k, cfg.normalize)
    y, rw, rid = block(xb, return_routing=True)
    x64 = _f64(xb)
    w, ids, n_near, n_diff = strict_route(x64, wr, rw.cpu().numpy(), rid.cpu().numpy(), cfg.k, cfg.normalize)
    print(f"{cfg.name}: near-tied tokens {n_near}, routed differently {n_diff} of {cfg.T}")
    ref = O.moe_ffn_block_grouped(x64, wr.astype(np.float64), *(_f64(t) for t in tb), cfg.E, cfg.k, cfg.H,
                                  cfg.F, cfg.normalize, routing=(w, ids))
    err = rms_rel_maxabs(y.float().cpu().numpy(), ref)
    assert err <= BLOCK_TOL, f"{cfg.name}: max-abs/rms {err:.3e}"
    assert ops.read_device_error() == 0
    return y


@pytest.mark.parametrize("cfg", [
    configs.BlockConfig("bf16_small", T=200, H=256, F=384, E=8, k=2, normalize=True, dtype="bf16"),
    configs.BlockConfig("bf16_fg", T=256, H=2048, F=768, E=128, k=8, normalize=False, dtype="bf16"),
    configs.BlockConfig("bf16_zipf", T=512, H=512, F=256, E=128, k=8, normalize=False, dtype="bf16", zipf=1.2),
    configs.c5(1), configs.c5(8), configs.c5(32), configs.c5(64),
], ids=lambda c: c.name)
def test_block_bf16(cfg):
    _block_check(cfg, seed=0)


def test_block_bf16_deterministic():
    cfg = configs.BlockConfig("det", T=300, H=512, F=256, E=16, k=4, normalize=False, dtype="bf16")
    x, wr, wu, wg, wd = configs.block_inputs_numpy(cfg, seed=2)
    block = ops.MoEFFNBlock(torch.from_numpy(wr).cuda(), *(_bf16(w) for w in (wu, wg, wd)), cfg.E, cfg.k, False)
    a = block(_bf16(x))
    b = block(_bf16(x))
    assert torch.equal(a, b)


def test_host_pipeline_equals_device_call():
    """ops.moe_ffn_host (chunked copies overlapping compute) returns exactly the
    single device call's output."""
    cfg = configs.BlockConfig("host_pipe", T=1000, H=512, F=256, E=16, k=4, normalize=True, dtype="bf16")
    x, wr, wu, wg, wd = configs.block_inputs_numpy(cfg, seed=4)
    block = ops.MoEFFNBlock(torch.from_numpy(wr).cuda(), *(_bf16(w) for w in (wu, wg, wd)), cfg.E, cfg.k, True)
    xb = _bf16(x)
    ref = block(xb)
    x_host = xb.cpu().pin_memory()
    y_host = torch.empty((cfg.T, cfg.H), dtype=torch.float32).pin_memory()
    for chunks in (1, 3, 7):
        y_host.zero_()
        ops.moe_ffn_host(block, x_host, y_host, chunks=chunks)
        torch.cuda.synchronize()
        assert torch.equal(y_host, ref.cpu())


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_host_pipeline_batches_equal_device_calls(depth):
    """ops.HostPipeline: a stream of different batches, copies of neighbouring
    batches overlapping compute, each equal bit for bit to one device call;
    host buffers reused across batches once their event completed."""
    cfg = configs.BlockConfig("host_stream", T=700, H=512, F=256, E=16, k=4, normalize=False, dtype="bf16")
    _, wr, wu, wg, wd = configs.block_inputs_numpy(cfg, seed=6)
    block = ops.MoEFFNBlock(torch.from_numpy(wr).cuda(), *(_bf16(w) for w in (wu, wg, wd)), cfg.E, cfg.k, False)
    pipe = ops.HostPipeline(block, cfg.T, cfg.H, torch.bfloat16, depth=depth)
    n_batches = 7
    xs = [torch.randn(cfg.T, cfg.H, generator=torch.Generator().manual_seed(i)).bfloat16().pin_memory()
          for i in range(n_batches)]
    refs = [block(x.cuda()).cpu() for x in xs]
    ys = [torch.empty((cfg.T, cfg.H), dtype=torch.float32).pin_memory() for _ in range(n_batches)]
    events = [pipe.submit(xs[i], ys[i]) for i in range(n_batches)]
    for i in range(n_batches):
        events[i].synchronize()
        assert torch.equal(ys[i], refs[i]), f"batch {i}"
    assert ops.read_device_error() == 0
