"""Decode-sized blocks (k*T <= E): the weight-streaming path vs the oracle.

Both forms of the path run: the single cooperative kernel (default) and the
five staged launches (FRANK_DECODE_FUSED=0); they execute the same
arithmetic in the same order, so their outputs must be bit-identical.  The
cases cover one token, ragged n_embd / n_ff (not multiples of the
column slices of the row groups), k*T == E, more rows per expert than one
pass stages (T > 8), and wide rows (n_embd = n_ff = 4096, and the
Mixtral-8x7B shapes: one weight row of 28 KB per down item).

The oracle (float64, moe_oracle.moe_ffn_block_grouped) runs with its own
routing under the strict tier (tests/utils.py ``strict_routing``: ids equal
the oracle's top-k on float64 logits except on tokens whose k-th/(k+1)-th
gap is below the fp32 accumulation bound), restricted to the experts routed
to.  Tolerance: max-abs <= 2e-2 x output RMS (bf16 h).
"""

import numpy as np
import pytest
import torch

from frank_b200 import configs, ops
from oracle import moe_oracle as O
from tests.utils import rms_rel_maxabs, strict_route

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _oracle_on_active(x, wr, wu, wg, wd, cfg, rw, rid):
    """moe_ffn_block_grouped restricted to the routed experts (ids remapped)."""
    act = np.unique(rid)
    remap = np.full(cfg.E, -1, dtype=np.int32)
    remap[act] = np.arange(act.size, dtype=np.int32)
    sl = torch.from_numpy(act).cuda()
    wu_a, wg_a, wd_a = (_f64(w.index_select(2, sl)) for w in (wu, wg, wd))
    return O.moe_ffn_block_grouped(_f64(x), wr.double().cpu().numpy(), wu_a, wg_a, wd_a, act.size, cfg.k, cfg.H,
                                   cfg.F, cfg.normalize, routing=(rw.astype(np.float64), remap[rid]))


def _run(block, x, fused, monkeypatch):
    monkeypatch.setenv("FRANK_DECODE_FUSED", "1" if fused else "0")
    y, rw, rid = block(x, return_routing=True)
    torch.cuda.synchronize()
    return y, rw.cpu().numpy(), rid.cpu().numpy()


@pytest.mark.parametrize("cfg", [
    configs.c5(1),
    configs.c5(16),                                                            # k*T == E
    configs.BlockConfig("ragged", T=3, H=528, F=272, E=64, k=6, normalize=True, dtype="bf16"),
    configs.BlockConfig("odd_tokens", T=5, H=1024, F=1536, E=40, k=8, normalize=False, dtype="bf16"),
    configs.BlockConfig("many_rows", T=12, H=256, F=512, E=16, k=1, normalize=False, dtype="bf16", zipf=3.0),
    configs.BlockConfig("wide", T=1, H=4096, F=4096, E=8, k=2, normalize=False, dtype="bf16"),
    configs.BlockConfig("mixtral_decode", T=2, H=4096, F=14336, E=8, k=2, normalize=False, dtype="bf16"),
], ids=lambda c: c.name)
def test_decode_block(cfg, monkeypatch):
    assert cfg.k * cfg.T <= cfg.E  # the decode path's condition
    x, wr, wu, wg, wd = configs.block_inputs_torch(cfg, "cuda", seed=11)
    block = ops.MoEFFNBlock(wr, wu, wg, wd, cfg.E, cfg.k, cfg.normalize)
    y1, rw, rid = _run(block, x, True, monkeypatch)
    y0, rw0, rid0 = _run(block, x, False, monkeypatch)
    assert np.array_equal(rid, rid0) and np.array_equal(rw, rw0)
    assert torch.equal(y1, y0), "fused and staged decode differ"
    w, ids, n_near, n_diff = strict_route(_f64(x), wr.cpu().numpy(), rw, rid, cfg.k, cfg.normalize)
    print(f"{cfg.name}: near-tied tokens {n_near}, routed differently {n_diff} of {cfg.T}")
    ref = _oracle_on_active(x, wr, wu, wg, wd, cfg, w, ids)
    err = rms_rel_maxabs(y1.float().cpu().numpy(), ref)
    assert err <= TOL, f"{cfg.name}: max-abs/rms {err:.3e}"
    assert ops.read_device_error() == 0


def test_decode_repeated_calls_identical(monkeypatch):
    """The fused kernel's grid-barrier counter is reset per call: many calls in
    a row give the same bits."""
    cfg = configs.c5(4)
    x, wr, wu, wg, wd = configs.block_inputs_torch(cfg, "cuda", seed=3)
    block = ops.MoEFFNBlock(wr, wu, wg, wd, cfg.E, cfg.k, cfg.normalize)
    monkeypatch.setenv("FRANK_DECODE_FUSED", "1")
    first = block(x)
    for _ in range(20):
        assert torch.equal(block(x), first)
    assert ops.read_device_error() == 0


def test_decode_leaves_workspace_header_zero(monkeypatch):
    """The fused kernel's grid-barrier counters live in the workspace header:
    zeroed once at allocation, left zero by every call (no per-call reset),
    also across a prefill-sized call that reuses the same workspace."""
    cfg = configs.c5(2)
    x, wr, wu, wg, wd = configs.block_inputs_torch(cfg, "cuda", seed=5)
    block = ops.MoEFFNBlock(wr, wu, wg, wd, cfg.E, cfg.k, cfg.normalize)
    monkeypatch.setenv("FRANK_DECODE_FUSED", "1")
    first = block(x)
    big = torch.randn(300, cfg.H, device="cuda").bfloat16()
    block(big)  # tensor-core path on the same (grown) workspace
    for _ in range(5):
        assert torch.equal(block(x), first)
    torch.cuda.synchronize()
    assert int(block._ws[:ops.WORKSPACE_HEADER_BYTES].count_nonzero()) == 0
    assert ops.read_device_error() == 0


def test_graphed_host_step_equals_device_call():
    """ops.GraphedHostMoEFFN: host tokens in, block, host result out as one
    graph launch; bit-identical to a device call, across replays with new
    tokens."""
    cfg = configs.c5(4)
    x, wr, wu, wg, wd = configs.block_inputs_torch(cfg, "cuda", seed=8)
    block = ops.MoEFFNBlock(wr, wu, wg, wd, cfg.E, cfg.k, cfg.normalize)
    g = ops.GraphedHostMoEFFN(block, cfg.T)
    for seed in (1, 2, 3):
        xs = torch.randn(cfg.T, cfg.H, generator=torch.Generator().manual_seed(seed)).bfloat16()
        g.x_host.copy_(xs)
        g.replay().synchronize()
        assert torch.equal(g.y_host, block(xs.cuda()).cpu())
    assert ops.read_device_error() == 0
