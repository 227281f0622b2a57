"""rms_norm and the MoE FFN sub-layer (residual + moe_ffn_block(rms_norm(residual)))
through the reference-shaped module and the torch API, against the reference's
own outputs (tests/golden/rmsnorm_*, sublayer_*: oracles/normalization.py and
oracles/moe.py composed as oracles/transformer_layer.py:107-124) and the
oracle restatement.

Tolerances: fp32 path rtol 1e-4 / atol 1e-5 (the reference's component
tests); bf16 path max-abs of the block part <= 2e-2 x its RMS, with the GPU's
routing handed to the oracle so near ties cannot swap experts.
"""

import numpy as np
import pytest
import torch

from frank_b200 import configs, ops
from oracle import moe_oracle as O
from tests.utils import assert_close, golden_names, load_golden, rms_rel_maxabs

pytestmark = pytest.mark.gpu

BLOCK_TOL = 2e-2


def _sub_args(g):
    return (g["residual"], g["ffn_norm_w"], float(g["rms_eps"]), g["gate_inp_w"], g["up_exps_w"], g["gate_exps_w"],
            g["down_exps_w"], int(g["n_expert"]), int(g["n_expert_used"]), int(g["n_embd"]), int(g["n_ff"]),
            bool(g["normalize_weights"]))


@pytest.mark.parametrize("name", golden_names("rmsnorm_"))
def test_rms_norm_golden(moe_ffn_module, name):
    g = load_golden(name)
    y = moe_ffn_module.rms_norm(g["input"], g["weight"], float(g["eps"]))
    assert y.dtype == np.float32 and y.shape == g["expected"].shape
    assert_close(y, g["expected"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", golden_names("sublayer_"))
def test_sublayer_golden(moe_ffn_module, name):
    g = load_golden(name)
    y = moe_ffn_module.moe_ffn_sublayer(*_sub_args(g))
    assert y.dtype == np.float32 and y.shape == g["expected"].shape
    assert_close(y, g["expected"], rtol=1e-4, atol=1e-5)


def _bf16_case(cfg, seed, in_place=False):
    x, wr, wu, wg, wd = configs.block_inputs_torch(cfg, "cuda", seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 7)
    residual = torch.randn((cfg.T, cfg.H), device="cuda", generator=g) * 2
    nw = 1 + 0.1 * torch.randn(cfg.H, device="cuda", generator=g)
    block = ops.MoEFFNBlock(wr, wu, wg, wd, cfg.E, cfg.k, cfg.normalize)
    eps = 1e-5
    if in_place:
        r0 = residual.clone()
        y, rw, rid = block.sublayer(residual, nw, eps, out=residual, return_routing=True)
        assert y.data_ptr() == residual.data_ptr()
        residual = r0
    else:
        y, rw, rid = block.sublayer(residual, nw, eps, return_routing=True)
    torch.cuda.synchronize()
    # oracle: rms_norm in fp32, tokens rounded to bf16 as the block consumes them
    r64 = residual.double().cpu().numpy()
    xn = ops.rms_norm(residual, nw, eps, out_dtype=torch.bfloat16)
    act = np.unique(rid.cpu().numpy())
    remap = np.full(cfg.E, -1, dtype=np.int32)
    remap[act] = np.arange(act.size, dtype=np.int32)
    sl = torch.from_numpy(act).cuda()
    wsel = [w.index_select(2, sl).double().cpu().numpy() for w in (wu, wg, wd)]
    moe = O.moe_ffn_block_grouped(xn.double().cpu().numpy(), wr.double().cpu().numpy(), *wsel, act.size, cfg.k,
                                  cfg.H, cfg.F, cfg.normalize,
                                  routing=(rw.cpu().numpy().astype(np.float64), remap[rid.cpu().numpy()]))
    got_moe = y.double().cpu().numpy() - r64
    assert rms_rel_maxabs(got_moe, moe) <= BLOCK_TOL
    # the residual add itself is exact up to one fp32 rounding of (r + moe)
    assert np.max(np.abs(y.double().cpu().numpy() - (r64 + moe))) <= 2e-2 * np.sqrt(np.mean(moe * moe)) + 1e-6
    # rms_norm on the GPU matches the oracle restatement
    xn_ref = O.rms_norm(residual.cpu().numpy(), nw.cpu().numpy(), eps)
    assert_close(ops.rms_norm(residual, nw, eps).cpu().numpy(), xn_ref, rtol=2e-6, atol=1e-6)
    assert ops.read_device_error() == 0
    return y


@pytest.mark.parametrize("cfg", [
    configs.BlockConfig("sub_prefill", T=300, H=512, F=256, E=16, k=4, normalize=False, dtype="bf16"),
    configs.BlockConfig("sub_renorm", T=129, H=256, F=384, E=8, k=2, normalize=True, dtype="bf16"),
    configs.c5(1),
    configs.c5(8),
], ids=lambda c: c.name)
def test_sublayer_bf16(cfg):
    _bf16_case(cfg, seed=3)


@pytest.mark.parametrize("fused", ["1", "0"])
def test_sublayer_in_place_equals_out_of_place(fused, monkeypatch):
    """out = residual (the in-place update a layer stack uses) gives the same
    bits as a separate output, on the tensor-core path and both decode forms."""
    monkeypatch.setenv("FRANK_DECODE_FUSED", fused)
    for cfg in (configs.BlockConfig("sub_ip", T=200, H=256, F=128, E=8, k=2, normalize=False, dtype="bf16"),
                configs.c5(2)):
        a = _bf16_case(cfg, seed=5)
        b = _bf16_case(cfg, seed=5, in_place=True)
        assert torch.equal(a, b)
