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
    oracles/transformer_layer.py:107-124 does;
  * whole MoE transformer layers of the toy model (transformer_layer_moe,
    oracles/transformer_layer.py:14-124) on the token batches of the toy
    model's prefill tests, with the attention half's residual stored beside.

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


TOY = dict(vocab_size=256, n_embd=64, n_head=4, n_head_kv=2, head_dim=16, n_ff=128, n_expert=4, n_expert_used=2,
           n_layers=2, rms_eps=1e-5, rope_freq_base=10000.0)


def toy_params(seed=42):
    """The toy MoE model's parameters, drawn in the order of the reference's
    generator (tests/models/test_toy_llm.py:49-124: default_rng(42), model
    tensors, then per layer the norms, attention projections, zero biases and
    the MoE weights) so the layers below are the toy model's own layers."""
    rng = np.random.default_rng(seed)
    c = TOY
    n = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    p = {"token_embd.weight": n(c["vocab_size"], c["n_embd"]), "output_norm.weight": n(c["n_embd"]),
         "output.weight": n(c["n_embd"], c["vocab_size"])}
    kv = c["n_head_kv"] * c["head_dim"]
    for i in range(c["n_layers"]):
        b = f"blk.{i}"
        p[f"{b}.attn_norm.weight"] = n(c["n_embd"])
        p[f"{b}.ffn_norm.weight"] = n(c["n_embd"])
        p[f"{b}.attn_q.weight"] = n(c["n_embd"], c["n_embd"])
        p[f"{b}.attn_k.weight"] = n(c["n_embd"], kv)
        p[f"{b}.attn_v.weight"] = n(c["n_embd"], kv)
        p[f"{b}.attn_output.weight"] = n(c["n_embd"], c["n_embd"])
        p[f"{b}.attn_q.bias"] = np.zeros(c["n_embd"], dtype=np.float32)
        p[f"{b}.attn_k.bias"] = np.zeros(kv, dtype=np.float32)
        p[f"{b}.attn_v.bias"] = np.zeros(kv, dtype=np.float32)
        p[f"{b}.attn_output.bias"] = np.zeros(c["n_embd"], dtype=np.float32)
        p[f"{b}.ffn_gate_inp.weight"] = n(c["n_expert"], c["n_embd"])
        p[f"{b}.ffn_up_exps.weight"] = n(c["n_ff"], c["n_embd"], c["n_expert"])
        p[f"{b}.ffn_gate_exps.weight"] = n(c["n_ff"], c["n_embd"], c["n_expert"])
        p[f"{b}.ffn_down_exps.weight"] = n(c["n_embd"], c["n_ff"], c["n_expert"])
    return p


# the token batches of the toy model's prefill tests (test_toy_llm.py:677-801)
TOY_BATCHES = {"tok4": np.array([[1, 2, 3, 4]]), "batch2": np.array([[10, 20, 30], [40, 50, 60]]),
               "tok8": np.arange(1, 9).reshape(1, 8)}


def toy_layer_cases(ref_layer, ref_norm, ref_attn):
    """Whole MoE transformer layers of the toy model (layers 0 and 1, the
    layer-1 input being layer 0's oracle output), each as the reference's
    transformer_layer_moe computes it (oracles/transformer_layer.py:14-124),
    plus the attention half's residual (input + attention, :74-104), which the
    GPU test feeds to the MoE FFN sub-layer."""
    c = TOY
    p = toy_params()
    out = []
    for tag, tokens in TOY_BATCHES.items():
        batch, seq = tokens.shape
        pos = np.tile(np.arange(seq, dtype=np.int64), (batch, 1))
        h = p["token_embd.weight"][tokens]
        for li in range(c["n_layers"]):
            b = f"blk.{li}"
            normed = ref_norm.rms_norm(h.reshape(-1, c["n_embd"]), p[f"{b}.attn_norm.weight"], c["rms_eps"])
            attn = ref_attn.attention_block(normed.reshape(batch, seq, c["n_embd"]), pos, p[f"{b}.attn_q.weight"],
                                            p[f"{b}.attn_k.weight"], p[f"{b}.attn_v.weight"],
                                            p[f"{b}.attn_output.weight"], p[f"{b}.attn_q.bias"],
                                            p[f"{b}.attn_k.bias"], p[f"{b}.attn_v.bias"],
                                            p[f"{b}.attn_output.bias"], False, c["n_head"], c["n_head_kv"],
                                            c["n_embd"], c["rope_freq_base"], 1.0)
            resid1 = h + attn
            y = ref_layer.transformer_layer_moe(h, pos, p, li, c["n_head"], c["n_head_kv"], c["n_embd"], c["n_ff"],
                                                c["n_expert"], c["n_expert_used"], rms_eps=c["rms_eps"],
                                                rope_freq_base=c["rope_freq_base"])
            out.append((f"layer_toy_{tag}_l{li}", dict(
                layer_input=h.astype(np.float32), residual1=resid1.astype(np.float32),
                ffn_norm_w=p[f"{b}.ffn_norm.weight"], rms_eps=np.float32(c["rms_eps"]),
                gate_inp_w=p[f"{b}.ffn_gate_inp.weight"], up_exps_w=p[f"{b}.ffn_up_exps.weight"],
                gate_exps_w=p[f"{b}.ffn_gate_exps.weight"], down_exps_w=p[f"{b}.ffn_down_exps.weight"],
                n_expert=c["n_expert"], n_expert_used=c["n_expert_used"], n_embd=c["n_embd"], n_ff=c["n_ff"],
                normalize_weights=False, expected=y.astype(np.float32))))
            h = y
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
    from oracles import attention as ref_attn
    from oracles import transformer_layer as ref_layer

    for name, arrays in toy_layer_cases(ref_layer, ref_norm, ref_attn):
        if keep(name):
            np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print("wrote", len(list(HERE.glob("*.npz"))), "fixtures to", HERE)


if __name__ == "__main__":
    main()
