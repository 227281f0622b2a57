"""Generate golden fixtures by running the reference's own NumPy oracles.

Run in a checkout that has the frank-models sources (the reference):

    python tests/golden/make_golden.py --reference <path to frank-models>

It imports ``oracles/moe.py`` and ``oracles/activation.py`` from that tree,
evaluates them on seeded inputs and writes one ``.npz`` per case into this
directory (inputs and the reference outputs).  The committed fixtures pin the
CPU restatement in ``oracle/`` (tests/test_oracle_golden.py) and the CUDA
path (the gpu-marked parity tests) to the reference's own numbers; nothing
at test time needs the reference tree.

Cases
  * the inputs of the reference's component tests for mul_mat_id
    (tests/components/test_mul_mat_id.py:15-85), moe_ffn_block
    (test_moe_ffn_block.py:20-196) and swiglu (test_swiglu.py:15-59):
    same seeds, shapes, fixed ids and legacy ``np.random.seed`` + ``randn``
    draws;
  * the fp32 headline configuration (T=32, H=64, F=128, E=8, k=2, renorm);
  * small shapes of the fine-grained / decode families (E=128, k=8) with
    reduced H and F so the literal oracle stays cheap;
  * rms_norm (oracles/normalization.py) and the MoE FFN sub-layer, composed
    from the reference's rms_norm and moe_ffn_block exactly as
    oracles/transformer_layer.py:107-124 does.

``--only PREFIX`` writes just the cases whose names start with PREFIX.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "frank-models_b200"))


def _randn(*shape, scale=0.1):
    return np.random.randn(*shape).astype(np.float32) * scale


def mul_mat_id_cases():
    """(name, weights, input, ids) following test_mul_mat_id.py:15-85."""
    out = []
    np.random.seed(42)
    w = _randn(4, 3, 8)
    x = _randn(3, 1, 2)
    out.append(("mmid_single_expert", w, x, np.array([[0, 3]], dtype=np.int32)))
    np.random.seed(123)
    w = _randn(8, 4, 8)
    x = _randn(4, 2, 4)
    out.append(("mmid_two_experts", w, x, np.array([[0, 1, 2, 3], [4, 5, 6, 7]], dtype=np.int32)))
    np.random.seed(456)
    w = _randn(6, 4, 4)
    x = _randn(4, 1, 3)
    out.append(("mmid_same_expert", w, x, np.array([[2, 2, 2]], dtype=np.int32)))
    np.random.seed(789)
    w = _randn(64, 32, 8)
    x = _randn(32, 2, 16)
    ids = np.random.randint(0, 8, size=(2, 16), dtype=np.int32)
    out.append(("mmid_larger", w, x, ids))
    # extra: ragged expert load with empty experts, k=4 (duplicates allowed)
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((48, 40, 16)) * 0.1).astype(np.float32)
    x = (rng.standard_normal((40, 4, 37)) * 0.1).astype(np.float32)
    ids = rng.choice([1, 3, 3, 8, 15], size=(4, 37)).astype(np.int32)
    out.append(("mmid_ragged_k4", w, x, ids))
    return out


def moe_cases():
    """(name, inputs, E, k, H, F, normalize) following test_moe_ffn_block.py:20-196."""
    out = []
    for name, seed, (T, H, F), (E, k), norm in (
        ("moe_basic", 42, (4, 8, 16), (4, 2), False),
        ("moe_normalized", 123, (3, 8, 12), (4, 2), True),
        ("moe_single_expert", 456, (4, 8, 16), (8, 1), False),
        ("moe_mixtral_like", 789, (8, 32, 64), (8, 2), False),
    ):
        np.random.seed(seed)
        x = _randn(T, H)
        wr = _randn(E, H)
        wu = _randn(F, H, E)
        wg = _randn(F, H, E)
        wd = _randn(H, F, E)
        out.append((name, (x, wr, wu, wg, wd), E, k, H, F, norm))
    from frank_b200 import configs

    c1 = configs.C1
    out.append(("moe_c1_fp32", configs.block_inputs_numpy(c1, seed=0), c1.E, c1.k, c1.H, c1.F, c1.normalize))
    small_fg = configs.BlockConfig("fg_small", T=24, H=32, F=16, E=128, k=8, normalize=False, dtype="f32")
    out.append(("moe_fine_grained_small", configs.block_inputs_numpy(small_fg, seed=3), 128, 8, 32, 16, False))
    small_zipf = configs.BlockConfig("zipf_small", T=40, H=32, F=24, E=128, k=8, normalize=True, dtype="f32",
                                     zipf=1.2)
    out.append(("moe_zipf_small_norm", configs.block_inputs_numpy(small_zipf, seed=5), 128, 8, 32, 24, True))
    dec = configs.BlockConfig("decode_t1", T=1, H=32, F=16, E=128, k=8, normalize=False, dtype="f32")
    out.append(("moe_decode_t1", configs.block_inputs_numpy(dec, seed=0), 128, 8, 32, 16, False))
    return out


def swiglu_cases():
    """following test_swiglu.py:15-59."""
    out = []
    np.random.seed(42)
    out.append(("swiglu_random", np.random.randn(2, 4, 8).astype(np.float32),
                np.random.randn(2, 4, 8).astype(np.float32)))
    out.append(("swiglu_zeros", np.zeros((2, 4, 8), np.float32), np.zeros((2, 4, 8), np.float32)))
    np.random.seed(123)
    g = np.abs(np.random.randn(2, 4, 8).astype(np.float32)) + 0.1
    u = np.abs(np.random.randn(2, 4, 8).astype(np.float32)) + 0.1
    out.append(("swiglu_positive", g, u))
    np.random.seed(456)
    g = np.random.randn(2, 4, 8).astype(np.float32) * 10
    u = np.random.randn(2, 4, 8).astype(np.float32) * 10
    out.append(("swiglu_large", g, u))
    return out


def norm_cases():
    """rms_norm (oracles/normalization.py:10-43) and the MoE FFN sub-layer
    (oracles/transformer_layer.py:107-124): seeded residual streams, norm
    weights around 1, the block weights of moe_cases' shapes."""
    out = []
    rng = np.random.default_rng(21)
    for name, T, H in (("rmsnorm_small", 5, 64), ("rmsnorm_ragged", 7, 130)):
        x = rng.standard_normal((T, H), dtype=np.float32) * 3
        w = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        out.append((name, x, w, np.float32(1e-5)))
    return out


def sublayer_cases():
    out = []
    for name, seed, (T, H, F), (E, k), norm, eps in (
        ("sublayer_basic", 31, (6, 32, 48), (4, 2), False, 1e-5),
        ("sublayer_renorm", 32, (9, 64, 128), (8, 2), True, 1e-6),
        ("sublayer_fine_grained", 33, (12, 32, 16), (64, 6), False, 1e-5),
    ):
        rng = np.random.default_rng(seed)
        resid = rng.standard_normal((T, H), dtype=np.float32) * 2
        nw = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        wr = (rng.standard_normal((E, H)) * 0.1).astype(np.float32)
        wu = (rng.standard_normal((F, H, E)) * 0.1).astype(np.float32)
        wg = (rng.standard_normal((F, H, E)) * 0.1).astype(np.float32)
        wd = (rng.standard_normal((H, F, E)) * 0.1).astype(np.float32)
        out.append((name, (resid, nw, np.float32(eps), wr, wu, wg, wd), E, k, H, F, norm))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the frank-models source tree")
    ap.add_argument("--only", default="", help="write only the cases whose name starts with this prefix")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from oracles import activation as ref_act  # the reference's own oracle
    from oracles import moe as ref_moe
    from oracles import normalization as ref_norm

    def keep(name):
        return name.startswith(args.only)

    for name, w, x, ids in mul_mat_id_cases():
        if not keep(name):
            continue
        y = ref_moe.mul_mat_id(w, x, ids)
        np.savez_compressed(HERE / f"{name}.npz", weights=w, input=x, ids=ids, expected=y)
    for name, (x, wr, wu, wg, wd), E, k, H, F, norm in moe_cases():
        if not keep(name):
            continue
        y = ref_moe.moe_ffn_block(x, wr, wu, wg, wd, E, k, H, F, norm)
        np.savez_compressed(HERE / f"{name}.npz", input=x, gate_inp_w=wr, up_exps_w=wu, gate_exps_w=wg,
                            down_exps_w=wd, n_expert=E, n_expert_used=k, n_embd=H, n_ff=F,
                            normalize_weights=norm, expected=y)
    for name, g, u in swiglu_cases():
        if not keep(name):
            continue
        np.savez_compressed(HERE / f"{name}.npz", gate=g, up=u, expected=ref_act.swiglu(g, u))
    for name, x, w, eps in norm_cases():
        if not keep(name):
            continue
        np.savez_compressed(HERE / f"{name}.npz", input=x, weight=w, eps=eps,
                            expected=ref_norm.rms_norm(x, w, float(eps)))
    for name, (resid, nw, eps, wr, wu, wg, wd), E, k, H, F, norm in sublayer_cases():
        if not keep(name):
            continue
        # the sub-layer exactly as oracles/transformer_layer.py:107-124 composes it
        normed = ref_norm.rms_norm(resid, nw, float(eps))
        moe = ref_moe.moe_ffn_block(normed, wr, wu, wg, wd, E, k, H, F, norm)
        np.savez_compressed(HERE / f"{name}.npz", residual=resid, ffn_norm_w=nw, rms_eps=eps, gate_inp_w=wr,
                            up_exps_w=wu, gate_exps_w=wg, down_exps_w=wd, n_expert=E, n_expert_used=k, n_embd=H,
                            n_ff=F, normalize_weights=norm, expected=resid + moe)
    print("wrote", len(list(HERE.glob("*.npz"))), "fixtures to", HERE)


if __name__ == "__main__":
    main()
