"""The reference-facing surface: a module object whose methods have the names,
argument order and numpy-in/numpy-out behaviour of the IREE modules that the
reference's tests call.

Reference harness: tests/utils.py:171-223 (``IREEModule.invoke`` and
``__getattr__``: numpy arrays in, numpy arrays out after a synchronous
device->host copy), fixtures in tests/components/test_mul_mat_id.py:10-12,
test_moe_ffn_block.py:10-17, test_swiglu.py:10-12.

numpy inputs must be float32 (int32 for ids), as the fp32 MLIR components
require; they run the FFMA path and return numpy.  torch CUDA tensors run on
the current stream and return torch tensors (bf16 inputs take the tcgen05
path).
"""

from __future__ import annotations

import numpy as np
import torch

from . import ops


def _is_np(*xs) -> bool:
    return any(isinstance(x, np.ndarray) for x in xs)


def _dev(arr: np.ndarray, dtype: np.dtype, name: str) -> torch.Tensor:
    arr = np.ascontiguousarray(arr)
    if arr.dtype != dtype:
        raise ValueError(f"Unsupported dtype for {name}: {arr.dtype} (expected {np.dtype(dtype)})")
    return torch.from_numpy(arr).to(device="cuda", non_blocking=False)


def _host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.current_stream().synchronize()
    return t.cpu().numpy()


class B200Module:
    """Drop-in for the compiled ``moe_components`` / ``moe_ffn_components`` /
    ``activation_components`` modules."""

    def swiglu(self, gate, up):
        """@activation_components.swiglu(gate, up) -> gate * silu(up)."""
        if _is_np(gate, up):
            return _host(ops.swiglu(_dev(gate, np.float32, "gate"), _dev(up, np.float32, "up")))
        return ops.swiglu(gate, up)

    def mul_mat_id(self, weights, input, ids):
        """@moe_components.mul_mat_id(weights [O,I,E], input [I,k,T], ids [k,T] i32) -> [O,k,T]."""
        if _is_np(weights, input, ids):
            w = ops.PackedExperts.from_reference(_dev(weights, np.float32, "weights"), torch.float32)
            out = ops.mul_mat_id(w, _dev(input, np.float32, "input"), _dev(ids, np.int32, "ids"))
            return _host(out)
        return ops.mul_mat_id(weights, input, ids)

    def moe_ffn_block(self, input, gate_inp_w, up_exps_w, gate_exps_w, down_exps_w, n_expert, n_expert_used,
                      n_embd, n_ff, normalize_weights):
        """@moe_ffn_components.moe_ffn_block with the reference's ten arguments
        (moe_ffn_block.mlir:34-45) -> [T, n_embd]."""
        numpy_in = _is_np(input, gate_inp_w, up_exps_w, gate_exps_w, down_exps_w)
        if numpy_in:
            x = _dev(input, np.float32, "input")
            wr = _dev(gate_inp_w, np.float32, "gate_inp_w")
            wu = _dev(up_exps_w, np.float32, "up_exps_w")
            wg = _dev(gate_exps_w, np.float32, "gate_exps_w")
            wd = _dev(down_exps_w, np.float32, "down_exps_w")
            _check_block_shapes(x, wr, wu, wg, wd, n_expert, n_expert_used, n_embd, n_ff)
            # fresh uploads: pack directly instead of through the pointer-keyed cache
            wu, wg, wd = (ops.PackedExperts.from_reference(w, torch.float32) for w in (wu, wg, wd))
        else:
            x, wr, wu, wg, wd = input, gate_inp_w, up_exps_w, gate_exps_w, down_exps_w
        _check_block_shapes(x, wr, wu, wg, wd, n_expert, n_expert_used, n_embd, n_ff)
        block = ops.MoEFFNBlock(wr, wu, wg, wd, n_expert, n_expert_used, normalize_weights, dtype=x.dtype)
        y = block(x)
        return _host(y) if numpy_in else y

    def rms_norm(self, input, weight, eps):
        """@rms_norm_components.rms_norm_linalg(input [T, H], weight [H], eps)
        (components/normalization/rms_norm.mlir:18-80) -> [T, H] float32."""
        if _is_np(input, weight):
            return _host(ops.rms_norm(_dev(input, np.float32, "input"), _dev(weight, np.float32, "weight"), eps))
        return ops.rms_norm(input, weight, eps)

    # the reference module's exported name for the same function
    # (components/normalization/rms_norm.mlir:18, tests/components/test_rms_norm.py:22)
    rms_norm_linalg = rms_norm

    def moe_ffn_sublayer(self, residual, ffn_norm_w, rms_eps, gate_inp_w, up_exps_w, gate_exps_w, down_exps_w,
                         n_expert, n_expert_used, n_embd, n_ff, normalize_weights):
        """The MoE FFN sub-layer of the MoE transformer layer
        (transformer_layer_moe_prefill.mlir:211-245, decode :228-256,
        oracles/transformer_layer.py:107-124):
        residual + moe_ffn_block(rms_norm(residual, ffn_norm_w, rms_eps), ...)
        -> [T, n_embd] float32.  numpy in: fp32 FFMA path; torch CUDA in: the
        block runs in the expert weights' dtype (bf16: tcgen05)."""
        numpy_in = _is_np(residual, ffn_norm_w, gate_inp_w, up_exps_w, gate_exps_w, down_exps_w)
        if numpy_in:
            r = _dev(residual, np.float32, "residual")
            nw = _dev(ffn_norm_w, np.float32, "ffn_norm_w")
            wr = _dev(gate_inp_w, np.float32, "gate_inp_w")
            wu, wg, wd = (ops.PackedExperts.from_reference(_dev(w, np.float32, name), torch.float32)
                          for w, name in ((up_exps_w, "up_exps_w"), (gate_exps_w, "gate_exps_w"),
                                          (down_exps_w, "down_exps_w")))
            dtype = torch.float32
        else:
            r, nw, wr, wu, wg, wd = residual, ffn_norm_w, gate_inp_w, up_exps_w, gate_exps_w, down_exps_w
            dtype = wu.packed.dtype if isinstance(wu, ops.PackedExperts) else wu.dtype
        _check_block_shapes(r, wr, wu, wg, wd, n_expert, n_expert_used, n_embd, n_ff)
        block = ops.MoEFFNBlock(wr, wu, wg, wd, n_expert, n_expert_used, normalize_weights, dtype=dtype)
        y = block.sublayer(r, nw, rms_eps)
        return _host(y) if numpy_in else y


def _check_block_shapes(x, wr, wu, wg, wd, E, k, H, F):
    def shp(t):
        return tuple(t.shape) if not isinstance(t, ops.PackedExperts) else None

    if tuple(x.shape[1:]) != (H,):
        raise ValueError(f"moe_ffn_block: input {tuple(x.shape)} does not have n_embd={H}")
    if tuple(wr.shape) != (E, H):
        raise ValueError(f"moe_ffn_block: gate_inp_w {tuple(wr.shape)} != [{E}, {H}]")
    for name, w, want in (("up_exps_w", wu, (F, H, E)), ("gate_exps_w", wg, (F, H, E)),
                          ("down_exps_w", wd, (H, F, E))):
        s = shp(w)
        if s is not None and s != want:
            raise ValueError(f"moe_ffn_block: {name} {s} != {list(want)}")
    if not (1 <= k <= E):
        raise ValueError(f"moe_ffn_block: n_expert_used={k} outside [1, n_expert={E}]")
