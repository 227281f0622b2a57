"""Binding of the reference's GGUF-style parameter names to the MoE FFN path.

The reference names the MoE tensors of layer i

    blk.{i}.ffn_norm.weight        [H]         (the sub-layer's rms_norm weight)
    blk.{i}.ffn_gate_inp.weight    [E, H]      (router)
    blk.{i}.ffn_up_exps.weight     [F, H, E]
    blk.{i}.ffn_gate_exps.weight   [F, H, E]
    blk.{i}.ffn_down_exps.weight   [H, F, E]

(models/llm/mixtral/params.mlir:361-383, the toy model's parameter dict in
tests/models/test_toy_llm.py:111-124, read back by
oracles/transformer_layer.py:64-77).  :func:`moe_layer_from_params` checks
the names and shapes on the host, uploads each tensor once and packs the
expert tensors straight into the kernels' [E, O, I] layout in chunks of
output rows, so that a layer needs at most one chunk of staging memory
beside its packed weights.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Mapping

import numpy as np
import torch

from . import ops

_SUFFIXES = ("ffn_gate_inp.weight", "ffn_up_exps.weight", "ffn_gate_exps.weight", "ffn_down_exps.weight")


def param_names(layer_idx: int) -> dict[str, str]:
    """The reference's names of layer ``layer_idx``'s MoE tensors."""
    p = f"blk.{layer_idx}."
    return {"norm": p + "ffn_norm.weight", "router": p + "ffn_gate_inp.weight", "up": p + "ffn_up_exps.weight",
            "gate": p + "ffn_gate_exps.weight", "down": p + "ffn_down_exps.weight"}


@dataclass(frozen=True)
class MoEShapes:
    n_expert: int
    n_embd: int
    n_ff: int
    has_norm: bool


def _shape(a) -> tuple:
    return tuple(int(d) for d in a.shape)


def moe_param_shapes(params: Mapping[str, object], layer_idx: int) -> MoEShapes:
    """Validate the MoE tensors of one layer (host only, no device work) and
    return their dimensions.  Raises KeyError for a missing name and
    ValueError for inconsistent shapes."""
    n = param_names(layer_idx)
    for key in ("router", "up", "gate", "down"):
        if n[key] not in params:
            raise KeyError(f"missing parameter {n[key]!r}")
    E, H = _shape(params[n["router"]])
    up = _shape(params[n["up"]])
    if len(up) != 3 or up[1:] != (H, E):
        raise ValueError(f"{n['up']}: shape {list(up)} is not [n_ff, {H}, {E}]")
    F = up[0]
    if _shape(params[n["gate"]]) != (F, H, E):
        raise ValueError(f"{n['gate']}: shape {list(_shape(params[n['gate']]))} != [{F}, {H}, {E}]")
    if _shape(params[n["down"]]) != (H, F, E):
        raise ValueError(f"{n['down']}: shape {list(_shape(params[n['down']]))} != [{H}, {F}, {E}]")
    has_norm = n["norm"] in params
    if has_norm and _shape(params[n["norm"]]) != (H,):
        raise ValueError(f"{n['norm']}: shape {list(_shape(params[n['norm']]))} != [{H}]")
    return MoEShapes(E, H, F, has_norm)


def _to_device(a, device, dtype=torch.float32) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=device, dtype=dtype).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device=device, dtype=dtype)


def pack_reference_experts(w_oie, dtype: torch.dtype, device, chunk_bytes: int = 256 << 20) -> ops.PackedExperts:
    """[O, I, E] reference-layout expert tensor (numpy or torch, any device)
    -> PackedExperts [E, O, I] in ``dtype`` on ``device``, uploading and
    packing at most ``chunk_bytes`` of fp32 rows at a time."""
    O, I, E = _shape(w_oie)
    packed = torch.empty((E, O, I), dtype=dtype, device=device)
    rows = max(1, chunk_bytes // max(1, I * E * 4))
    for o0 in range(0, O, rows):
        o1 = min(O, o0 + rows)
        part = _to_device(w_oie[o0:o1], device)
        packed[:, o0:o1, :].copy_(ops.prepack_experts(part, dtype))
    return ops.PackedExperts(packed)


class MoELayer:
    """One layer's MoE FFN: the packed block and (when present) the
    sub-layer's rms_norm weight."""

    def __init__(self, block: ops.MoEFFNBlock, ffn_norm_w: torch.Tensor | None):
        self.block = block
        self.ffn_norm_w = ffn_norm_w

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """moe_ffn_block on tokens x [T, H] (the block's compute dtype)."""
        return self.block(x, out=out)

    def sublayer(self, residual: torch.Tensor, rms_eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
        """residual + moe_ffn_block(rms_norm(residual)) (oracles/transformer_layer.py:107-124)."""
        if self.ffn_norm_w is None:
            raise KeyError("this layer's parameters carry no ffn_norm.weight")
        return self.block.sublayer(residual, self.ffn_norm_w, rms_eps, out=out)


def moe_layer_from_params(params: Mapping[str, object], layer_idx: int, n_expert_used: int,
                          normalize_weights: bool = False, dtype: torch.dtype = torch.bfloat16, device=None,
                          chunk_bytes: int = 256 << 20) -> MoELayer:
    """Build layer ``layer_idx``'s MoE FFN from a name -> array mapping
    (numpy or torch; the reference's fp32 tensors).  Expert weights are packed
    to ``dtype`` (bf16: tensor-core path; fp32: FFMA path); the router and
    the norm weight stay fp32."""
    shapes = moe_param_shapes(params, layer_idx)
    if not (1 <= n_expert_used <= shapes.n_expert):
        raise ValueError(f"n_expert_used={n_expert_used} outside [1, {shapes.n_expert}]")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    n = param_names(layer_idx)
    wr = _to_device(params[n["router"]], dev)
    wu, wg, wd = (pack_reference_experts(params[n[key]], dtype, dev, chunk_bytes) for key in ("up", "gate", "down"))
    block = ops.MoEFFNBlock(wr, wu, wg, wd, shapes.n_expert, n_expert_used, normalize_weights, dtype=dtype)
    norm = _to_device(params[n["norm"]], dev) if shapes.has_norm else None
    return MoELayer(block, norm)


def moe_layers_from_params(params: Mapping[str, object], n_layers: int, n_expert_used: int, **kw) -> list[MoELayer]:
    """:func:`moe_layer_from_params` for layers 0 .. n_layers-1."""
    return [moe_layer_from_params(params, i, n_expert_used, **kw) for i in range(n_layers)]
