"""Parity at the stated shapes of the large configurations.

* C2: ``mul_mat_id`` alone, T=4096, 4096 -> 14336, E=8, k=2, distinct ids
  per token (the reference's mul_mat_id test pattern,
  tests/components/test_mul_mat_id.py:72-85, at full size), against the
  grouped oracle (oracles/moe.py:9-48) in float64 on the same bf16-rounded
  inputs: max-abs <= 1e-3 x output RMS.
* C3: the Mixtral-8x7B block, T=16384, H=4096, F=14336, E=8, k=2.  All
  16384 tokens' expert ids are held to the strict routing tier (equal to the
  oracle's top-k on float64 logits except on tokens whose k-th/(k+1)-th
  logit gap is below the fp32 accumulation bound; the count is printed),
  and the block output of a seeded 1024-token subset is checked against the
  oracle (oracles/moe.py:51-132) running its own routing: max-abs <= 2e-2 x
  output RMS.
* C4: the fine-grained block, T=8192, H=2048, F=768, E=128, k=8 with the
  Zipf(1.2) router skew, every token, same tiers.

The oracle runs on the host in float64, one expert's weights converted at a
time.  These cases exercise what small shapes cannot: the tensor-core
router at T=8192, experts with a handful of rows next to experts with
thousands, swapped tiles beside full tiles, and the 470 MB ``[O,k,T]``
output transpose.
"""

import numpy as np
import pytest
import torch

from frank_b200 import configs, ops
from oracle import moe_oracle as O
from tests.utils import ExpertSlices, rms_rel_maxabs, strict_route

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

BLOCK_TOL = 2e-2
MMID_TOL = 1e-3


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def _near_tie_cap(T):
    # disagreements are allowed only on near-tied tokens, and must stay rare
    return max(4, T // 500)


def test_c2_mul_mat_id_full_size():
    cfg = configs.C2
    w, inp, ids = configs.mul_mat_id_inputs_numpy(cfg, seed=0)
    wb = torch.from_numpy(w).cuda().bfloat16()
    del w
    xb = torch.from_numpy(inp).cuda().bfloat16()
    idt = torch.from_numpy(ids).cuda()
    out = ops.mul_mat_id(wb, xb, idt)
    torch.cuda.synchronize()
    assert ops.read_device_error() == 0
    got = out.cpu().numpy()
    del out
    ref = O.mul_mat_id_grouped(ExpertSlices(wb.permute(2, 0, 1)), _f64(xb), ids)
    err = rms_rel_maxabs(got, ref)
    print(f"c2: max-abs/rms {err:.3e}")
    assert got.shape == (cfg.n_out, cfg.k, cfg.T)
    assert err <= MMID_TOL


def test_c3_mixtral_full_size():
    cfg = configs.C3
    dev = torch.device("cuda")
    wr, wu_p, wg_p, wd_p = configs.block_weights_packed_torch(cfg, dev, seed=0)
    x = configs.block_x_torch(cfg, dev, seed=0)
    block = ops.MoEFFNBlock(wr, ops.PackedExperts(wu_p), ops.PackedExperts(wg_p), ops.PackedExperts(wd_p), cfg.E,
                            cfg.k, cfg.normalize)
    y, rw, rid = block(x, return_routing=True)
    torch.cuda.synchronize()
    assert ops.read_device_error() == 0
    x64 = _f64(x)
    wr32 = wr.cpu().numpy()
    w, ids, n_near, n_diff = strict_route(x64, wr32, rw.cpu().numpy(), rid.cpu().numpy(), cfg.k, cfg.normalize)
    print(f"c3: near-tied tokens {n_near}, routed differently {n_diff} of {cfg.T}")
    assert n_diff <= _near_tie_cap(cfg.T)
    sel = np.sort(np.random.default_rng(0).choice(cfg.T, 1024, replace=False))
    ref = O.moe_ffn_block_grouped(x64[sel], wr32.astype(np.float64), ExpertSlices(wu_p), ExpertSlices(wg_p),
                                  ExpertSlices(wd_p), cfg.E, cfg.k, cfg.H, cfg.F, cfg.normalize,
                                  routing=(w[:, sel], ids[:, sel]))
    err = rms_rel_maxabs(y[torch.from_numpy(sel).to(dev)].float().cpu().numpy(), ref)
    print(f"c3: 1024-token subset max-abs/rms {err:.3e}")
    assert err <= BLOCK_TOL


def test_c4_fine_grained_full_size():
    cfg = configs.C4
    x, wr, wu, wg, wd = configs.block_inputs_torch(cfg, "cuda", seed=0)
    block = ops.MoEFFNBlock(wr, wu, wg, wd, cfg.E, cfg.k, cfg.normalize)
    y, rw, rid = block(x, return_routing=True)
    torch.cuda.synchronize()
    assert ops.read_device_error() == 0
    x64 = _f64(x)
    wr32 = wr.cpu().numpy()
    w, ids, n_near, n_diff = strict_route(x64, wr32, rw.cpu().numpy(), rid.cpu().numpy(), cfg.k, cfg.normalize)
    counts = np.bincount(ids.reshape(-1), minlength=cfg.E)
    print(f"c4: near-tied tokens {n_near}, routed differently {n_diff} of {cfg.T}; "
          f"rows per expert max {counts.max()} min {counts.min()}, {(counts < 64).sum()} experts below 64")
    assert n_diff <= _near_tie_cap(cfg.T)
    ref = O.moe_ffn_block_grouped(x64, wr32.astype(np.float64), ExpertSlices(wu.permute(2, 0, 1)),
                                  ExpertSlices(wg.permute(2, 0, 1)), ExpertSlices(wd.permute(2, 0, 1)), cfg.E,
                                  cfg.k, cfg.H, cfg.F, cfg.normalize, routing=(w, ids))
    err = rms_rel_maxabs(y.float().cpu().numpy(), ref)
    print(f"c4: max-abs/rms {err:.3e}")
    assert err <= BLOCK_TOL
