"""Thin, typed wrappers over the C ABI that take and return torch tensors.

Every function launches on the current torch CUDA stream and returns
without synchronising.  Buffers (outputs and workspaces) are allocated here
with torch and handed to the library, which never allocates.
"""

from __future__ import annotations

from collections import OrderedDict

import torch

from . import _lib

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}
WORKSPACE_HEADER_BYTES = 256  # FRANK_WORKSPACE_HEADER_BYTES


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32 or bfloat16") from None


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _cuda_contig(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a torch.Tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError(f"{name}: tensor must be on a CUDA device")
    return t.contiguous()


def num_sms() -> int:
    return _lib.load().frank_num_sms()


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """gate * silu(up) (components/activation/swiglu.mlir:16-51)."""
    gate = _cuda_contig(gate, "gate")
    up = _cuda_contig(up, "up")
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise ValueError(f"swiglu: gate {tuple(gate.shape)}/{gate.dtype} vs up {tuple(up.shape)}/{up.dtype}")
    out = torch.empty_like(gate)
    _lib.check(_lib.load().frank_swiglu(_dt(gate), _ptr(gate), _ptr(up), _ptr(out), gate.numel(), _stream()))
    return out


def softmax_topk(logits: torch.Tensor, k: int, normalize: bool):
    """Softmax over experts + top-k from fp32 logits [E, T] -> (w [k,T] f32, ids [k,T] i32)."""
    logits = _cuda_contig(logits, "logits")
    if logits.dtype != torch.float32 or logits.dim() != 2:
        raise ValueError("softmax_topk: logits must be fp32 [E, T]")
    E, T = logits.shape
    w = torch.empty((k, T), dtype=torch.float32, device=logits.device)
    ids = torch.empty((k, T), dtype=torch.int32, device=logits.device)
    _lib.check(_lib.load().frank_softmax_topk(_ptr(logits), T, E, k, int(bool(normalize)), _ptr(w), _ptr(ids),
                                              _stream()))
    return w, ids


def router_pack(wr: torch.Tensor) -> torch.Tensor:
    """The router weights prepared once (frank_router_pack): an fp32 copy of
    wr [E, H] followed by its exact three-term bf16 split, as a uint8 device
    tensor.  Pass it as ``pack=`` to :func:`router_topk`; blocks build it at
    construction."""
    wr = _cuda_contig(wr, "wr")
    E, H = wr.shape
    lib = _lib.load()
    pack = torch.empty(lib.frank_router_pack_size(E, H), dtype=torch.uint8, device=wr.device)
    _lib.check(lib.frank_router_pack(_dt(wr), _ptr(wr), E, H, _ptr(pack), _stream()))
    return pack


def router_topk(x: torch.Tensor, wr: torch.Tensor, k: int, normalize: bool, pack: torch.Tensor | None = None):
    """Router logits + softmax + top-k (+ renorm) -> (w [k,T] f32, ids [k,T] i32).
    ``pack``: optional :func:`router_pack` of ``wr`` (same results, no
    per-call split of the router weights)."""
    x = _cuda_contig(x, "x")
    wr = _cuda_contig(wr, "wr")
    T, H = x.shape
    E = wr.shape[0]
    if wr.shape[1] != H:
        raise ValueError(f"router_topk: wr {tuple(wr.shape)} does not match n_embd={H}")
    w = torch.empty((k, T), dtype=torch.float32, device=x.device)
    ids = torch.empty((k, T), dtype=torch.int32, device=x.device)
    lib = _lib.load()
    nbytes = lib.frank_router_scratch_bytes(_dt(x), T, H, E)
    scratch = torch.empty((nbytes + 3) // 4, dtype=torch.float32, device=x.device) if nbytes else None
    wr_dt, wr_ptr = (_lib.ROUTER_PACKED, _ptr(pack)) if pack is not None else (_dt(wr), _ptr(wr))
    _lib.check(lib.frank_router_topk(_dt(x), _ptr(x), wr_dt, wr_ptr, T, H, E, k, int(bool(normalize)),
                                     _ptr(w), _ptr(ids), _ptr(scratch), _stream()))
    return w, ids


def permute(ids: torch.Tensor, n_expert: int):
    """Stable expert permutation of ids [k, T] -> (sorted_slots, offsets, slot_pos, err_flag)."""
    ids = _cuda_contig(ids, "ids")
    if ids.dtype != torch.int32:
        raise TypeError("permute: ids must be int32")
    n = ids.numel()
    lib = _lib.load()
    dev = ids.device
    sorted_slots = torch.empty(n, dtype=torch.int32, device=dev)
    offsets = torch.empty(n_expert + 1, dtype=torch.int32, device=dev)
    slot_pos = torch.empty(n, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_bytes = lib.frank_permute_workspace_size(n, n_expert)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    _lib.check(lib.frank_permute(_ptr(ids), n, n_expert, _ptr(sorted_slots), _ptr(offsets), _ptr(slot_pos),
                                 _ptr(err), _ptr(ws), ws_bytes, _stream()))
    return sorted_slots, offsets, slot_pos, err


def prepack_experts(w_oie: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """[O, I, E] expert-innermost weights -> packed [E, O, I] in out_dtype."""
    w_oie = _cuda_contig(w_oie, "weights")
    if w_oie.dim() != 3:
        raise ValueError("prepack_experts: weights must be 3-D [n_out, n_in, n_expert]")
    O, I, E = w_oie.shape
    out = torch.empty((E, O, I), dtype=out_dtype, device=w_oie.device)
    _lib.check(_lib.load().frank_prepack_experts(_dt(w_oie), _ptr(w_oie), O, I, E, _DT[out_dtype], _ptr(out),
                                                 _stream()))
    return out


class PackedExperts:
    """Expert weights already in the packed [E, O, I] layout."""

    def __init__(self, packed: torch.Tensor):
        if packed.dim() != 3:
            raise ValueError("PackedExperts: expected [E, O, I]")
        self.packed = packed.contiguous()

    @classmethod
    def from_reference(cls, w_oie: torch.Tensor, dtype: torch.dtype) -> "PackedExperts":
        return cls(prepack_experts(w_oie, dtype))

    @property
    def n_expert(self):
        return self.packed.shape[0]

    @property
    def n_out(self):
        return self.packed.shape[1]

    @property
    def n_in(self):
        return self.packed.shape[2]


class _PackCache:
    """Prepacked weights keyed by (storage pointer, version, shape, dtypes):
    a weight tensor is packed once and reused until it is modified.  Each
    entry keeps its source tensor alive so that its address cannot be reused
    by another tensor while the entry exists."""

    def __init__(self, capacity: int = 24):
        self.cap = capacity
        self.d: OrderedDict = OrderedDict()

    def get(self, w: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        key = (w.data_ptr(), w._version, tuple(w.shape), tuple(w.stride()), w.dtype, dtype, w.device)
        hit = self.d.get(key)
        if hit is not None:
            self.d.move_to_end(key)
            return hit[1]
        p = prepack_experts(w, dtype)
        self.d[key] = (w, p)
        if len(self.d) > self.cap:
            self.d.popitem(last=False)
        return p


PACK_CACHE = _PackCache()


def _packed(w, dtype: torch.dtype, name: str) -> torch.Tensor:
    if isinstance(w, PackedExperts):
        if w.packed.dtype != dtype:
            raise TypeError(f"{name}: packed dtype {w.packed.dtype} != compute dtype {dtype}")
        return w.packed
    return PACK_CACHE.get(_cuda_contig(w, name), dtype)


def mul_mat_id(weights, inp: torch.Tensor, ids: torch.Tensor, check_ids: bool = True) -> torch.Tensor:
    """Expert-selected matmul (components/moe/mul_mat_id.mlir:22-120).

    weights: [O, I, E] (reference layout) or PackedExperts; inp [I, k, T];
    ids [k, T] int32.  Returns fp32 [O, k, T].  fp32 inputs run the FFMA
    path; bf16 inputs the tcgen05 path.  With check_ids, out-of-range ids
    raise FrankError(EIDS) (this synchronises the stream).
    """
    inp = _cuda_contig(inp, "input")
    ids = _cuda_contig(ids, "ids")
    dtype = inp.dtype
    wp = _packed(weights, dtype, "weights")
    E, O, I = wp.shape
    if inp.dim() != 3 or inp.shape[0] != I:
        raise ValueError(f"mul_mat_id: input {tuple(inp.shape)} does not match n_in={I}")
    k, T = inp.shape[1], inp.shape[2]
    if tuple(ids.shape) != (k, T) or ids.dtype != torch.int32:
        raise ValueError(f"mul_mat_id: ids must be int32 [{k}, {T}], got {tuple(ids.shape)} {ids.dtype}")
    lib = _lib.load()
    out = torch.empty((O, k, T), dtype=torch.float32, device=inp.device)
    err = torch.zeros(1, dtype=torch.int32, device=inp.device)
    ws_bytes = lib.frank_mul_mat_id_workspace_size(_dt(inp), O, I, E, k, T)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=inp.device)
    _lib.check(lib.frank_mul_mat_id(_dt(inp), _ptr(wp), _ptr(inp), _ptr(ids), O, I, E, k, T, _ptr(out), _ptr(err),
                                    _ptr(ws), ws_bytes, _stream()))
    if check_ids and int(err.item()) != 0:
        raise _lib.FrankError(_lib.EIDS, f"mul_mat_id: an expert id is outside [0, {E})")
    return out


class MoEFFNBlock:
    """The MoE FFN block with weights packed once and a reusable workspace.

    Mirrors @moe_ffn_components.moe_ffn_block (moe_ffn_block.mlir:34-209):
    the weights are given in the reference layouts (router [E, H], up/gate
    [F, H, E], down [H, F, E]) and packed at construction.  ``dtype`` is the
    compute dtype (bf16: tcgen05, fp32: FFMA); ``out_dtype`` the dtype of y
    (default fp32, the reference's output type).
    """

    def __init__(self, gate_inp_w, up_exps_w, gate_exps_w, down_exps_w, n_expert: int, n_expert_used: int,
                 normalize_weights: bool, dtype: torch.dtype = torch.bfloat16,
                 out_dtype: torch.dtype = torch.float32):
        if dtype not in _DT:
            raise TypeError(f"MoEFFNBlock: unsupported compute dtype {dtype}")
        if out_dtype not in _DT:
            raise TypeError(f"MoEFFNBlock: unsupported output dtype {out_dtype}")
        self.dtype = dtype
        self.out_dtype = out_dtype
        self.E = int(n_expert)
        self.k = int(n_expert_used)
        self.normalize = bool(normalize_weights)
        self.wr = _cuda_contig(gate_inp_w, "gate_inp_w")
        self.w_up = _packed(up_exps_w, dtype, "up_exps_w")
        self.w_gate = _packed(gate_exps_w, dtype, "gate_exps_w")
        self.w_down = _packed(down_exps_w, dtype, "down_exps_w")
        E, F, H = self.w_up.shape
        if E != self.E or tuple(self.w_gate.shape) != (E, F, H) or tuple(self.w_down.shape) != (E, H, F):
            raise ValueError("MoEFFNBlock: expert weight shapes disagree")
        if tuple(self.wr.shape) != (E, H):
            raise ValueError(f"MoEFFNBlock: gate_inp_w {tuple(self.wr.shape)} != [{E}, {H}]")
        self.H, self.F = H, F
        self._ws = None
        # router weights prepared once (fp32 copy + the tensor-core router's
        # exact bf16 split), passed as FRANK_ROUTER_PACKED
        self.wr_pack = router_pack(self.wr)

    def workspace_bytes(self, T: int) -> int:
        return _lib.load().frank_moe_ffn_block_workspace_size(_DT[self.dtype], T, self.H, self.F, self.E, self.k)

    def _workspace(self, T: int, device, need: int | None = None) -> torch.Tensor:
        need = self.workspace_bytes(T) if need is None else need
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            self._ws = torch.empty(max(need, WORKSPACE_HEADER_BYTES), dtype=torch.uint8, device=device)
            # the header (the decode kernel's barrier counters) starts at zero;
            # every call leaves it zero again
            self._ws[:WORKSPACE_HEADER_BYTES].zero_()
        return self._ws

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, return_routing: bool = False):
        x = _cuda_contig(x, "input")
        if x.dtype != self.dtype or x.dim() != 2 or x.shape[1] != self.H:
            raise ValueError(f"moe_ffn_block: input must be {self.dtype} [T, {self.H}], got {x.dtype} "
                             f"{tuple(x.shape)}")
        T = x.shape[0]
        if out is not None and (out.dtype != self.out_dtype or tuple(out.shape) != (T, self.H)
                                or not out.is_contiguous()):
            raise ValueError(f"moe_ffn_block: out must be contiguous {self.out_dtype} [{T}, {self.H}]")
        y = out if out is not None else torch.empty((T, self.H), dtype=self.out_dtype, device=x.device)
        rw = torch.empty((self.k, T), dtype=torch.float32, device=x.device) if return_routing else None
        rid = torch.empty((self.k, T), dtype=torch.int32, device=x.device) if return_routing else None
        ws = self._workspace(T, x.device)
        _lib.check(_lib.load().frank_moe_ffn_block(
            _DT[self.dtype], _ptr(x), _lib.ROUTER_PACKED, _ptr(self.wr_pack), _ptr(self.w_up), _ptr(self.w_gate),
            _ptr(self.w_down), T, self.E, self.k, self.H, self.F, int(self.normalize), _DT[self.out_dtype], _ptr(y), _ptr(rw), _ptr(rid),
            _ptr(ws), ws.numel(), _stream()))
        if return_routing:
            return y, rw, rid
        return y

    def sublayer(self, residual: torch.Tensor, ffn_norm_w: torch.Tensor, rms_eps: float,
                 out: torch.Tensor | None = None, return_routing: bool = False):
        """The MoE FFN sub-layer of the reference's MoE transformer layer
        (transformer_layer_moe_prefill.mlir:211-245, oracles/transformer_layer.py:107-124):
        ``residual + moe_ffn_block(rms_norm(residual, ffn_norm_w, rms_eps))``.
        residual: fp32 [T, H] on the GPU; ffn_norm_w: fp32 [H].  The normalised
        tokens are rounded to the block's compute dtype; the residual add is
        fused into the final sum over the k slots.  ``out`` (fp32 [T, H]) may
        be ``residual`` itself (in-place update)."""
        residual = _cuda_contig(residual, "residual")
        ffn_norm_w = _cuda_contig(ffn_norm_w, "ffn_norm_w")
        if residual.dtype != torch.float32 or residual.dim() != 2 or residual.shape[1] != self.H:
            raise ValueError(f"moe_ffn_sublayer: residual must be float32 [T, {self.H}], got {residual.dtype} "
                             f"{tuple(residual.shape)}")
        if ffn_norm_w.dtype != torch.float32 or tuple(ffn_norm_w.shape) != (self.H,):
            raise ValueError(f"moe_ffn_sublayer: ffn_norm_w must be float32 [{self.H}]")
        T = residual.shape[0]
        if out is not None and (out.dtype != torch.float32 or tuple(out.shape) != (T, self.H)
                                or not out.is_contiguous()):
            raise ValueError(f"moe_ffn_sublayer: out must be contiguous float32 [{T}, {self.H}]")
        y = out if out is not None else torch.empty((T, self.H), dtype=torch.float32, device=residual.device)
        rw = torch.empty((self.k, T), dtype=torch.float32, device=residual.device) if return_routing else None
        rid = torch.empty((self.k, T), dtype=torch.int32, device=residual.device) if return_routing else None
        lib = _lib.load()
        need = lib.frank_moe_ffn_sublayer_workspace_size(_DT[self.dtype], T, self.H, self.F, self.E, self.k)
        ws = self._workspace(T, residual.device, need)
        _lib.check(lib.frank_moe_ffn_sublayer(
            _DT[self.dtype], _ptr(residual), _ptr(ffn_norm_w), float(rms_eps), _lib.ROUTER_PACKED, _ptr(self.wr_pack),
            _ptr(self.w_up), _ptr(self.w_gate), _ptr(self.w_down), T, self.E, self.k, self.H, self.F,
            int(self.normalize), _ptr(y), _ptr(rw), _ptr(rid), _ptr(ws), ws.numel(), _stream()))
        if return_routing:
            return y, rw, rid
        return y


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out_dtype: torch.dtype = torch.float32,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """@rms_norm_components.rms_norm_linalg (components/normalization/rms_norm.mlir:18-80):
    (x / sqrt(mean(x^2, -1) + eps)) * weight for fp32 x [T, H], weight [H];
    the result in ``out_dtype`` (fp32 or bf16)."""
    x = _cuda_contig(x, "input")
    weight = _cuda_contig(weight, "weight")
    if x.dtype != torch.float32 or x.dim() != 2:
        raise ValueError(f"rms_norm: input must be float32 [T, H], got {x.dtype} {tuple(x.shape)}")
    if weight.dtype != torch.float32 or tuple(weight.shape) != (x.shape[1],):
        raise ValueError(f"rms_norm: weight must be float32 [{x.shape[1]}]")
    y = out if out is not None else torch.empty(tuple(x.shape), dtype=out_dtype, device=x.device)
    _lib.check(_lib.load().frank_rms_norm(_ptr(x), _ptr(weight), x.shape[0], x.shape[1], float(eps), _DT[y.dtype],
                                          _ptr(y), _stream()))
    return y


def moe_ffn_host(block, x_host: torch.Tensor, y_host: torch.Tensor, chunks: int = 4,
                 x_dev: torch.Tensor | None = None, y_dev: torch.Tensor | None = None,
                 order_copy_out: bool = True):
    """Run ``block`` (a :class:`MoEFFNBlock`, or any callable ``block(x, out=y)``
    over token rows) on host-resident tokens: x_host [T, H] -> y_host [T, H]
    (pinned host tensors).  The tokens are split into ``chunks`` pieces that
    flow through three streams -- host-to-device copy, the block on the
    current stream, device-to-host copy -- so the PCIe transfers of one chunk
    overlap the compute of its neighbours.  Tokens are independent in the
    block, so the result equals one call on all T tokens bit for bit.
    x_dev / y_dev: optional device staging buffers of the full size
    (allocated when absent).  No host synchronisation.  Returns a CUDA event
    that completes when y_host is written; with ``order_copy_out`` (default)
    the current stream is also ordered after it.  Without, the copies out of
    this call overlap whatever the caller enqueues next (e.g. the next call),
    and the caller waits on the event before reading y_host."""
    T, H = x_host.shape
    if not (x_host.is_pinned() and y_host.is_pinned()):
        raise ValueError("moe_ffn_host: x_host and y_host must be pinned host tensors")
    dev = torch.device("cuda", torch.cuda.current_device())
    x_dev = x_dev if x_dev is not None else torch.empty((T, H), dtype=x_host.dtype, device=dev)
    y_dev = y_dev if y_dev is not None else torch.empty((T, H), dtype=y_host.dtype, device=dev)
    chunks = max(1, min(int(chunks), T))
    bounds = [T * i // chunks for i in range(chunks + 1)]
    compute = torch.cuda.current_stream(dev)
    s_in, s_out = _host_streams(dev)
    s_in.wait_stream(compute)
    s_out.wait_stream(compute)
    for i in range(chunks):
        a, b = bounds[i], bounds[i + 1]
        if a == b:
            continue
        with torch.cuda.stream(s_in):
            x_dev[a:b].copy_(x_host[a:b], non_blocking=True)
        compute.wait_stream(s_in)
        block(x_dev[a:b], out=y_dev[a:b])
        s_out.wait_stream(compute)
        with torch.cuda.stream(s_out):
            y_host[a:b].copy_(y_dev[a:b], non_blocking=True)
    done = torch.cuda.Event()
    done.record(s_out)
    if order_copy_out:
        compute.wait_event(done)
    return done


class HostPipeline:
    """Streams batches of host-resident tokens through ``block`` (a
    :class:`MoEFFNBlock`, or any callable ``block(x, out=y)``) with copies in
    and out overlapping the neighbouring batches' compute.

    ``submit(x_host, y_host)`` enqueues, for one batch: the host-to-device
    copy of x_host [T, H] into one of ``depth`` device slots (on a copy
    stream, once the block call that last read the slot is done), the block
    on the current stream, and the device-to-host copy into y_host (on a
    second copy stream).  Batch i+1's input copy therefore runs during batch
    i's block, and batch i's output copy during batch i+1's block; every
    batch still moves its own inputs and result across PCIe.  Returns a CUDA
    event that completes when y_host is written; until then the caller keeps
    x_host and y_host alive and does not modify them.  Pinned host tensors
    only; no host synchronisation.  The result of each batch equals one
    block call on the same tokens, bit for bit."""

    def __init__(self, block, T: int, H: int, x_dtype: torch.dtype, y_dtype: torch.dtype = torch.float32,
                 depth: int = 2, device=None):
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.block = block
        self.T, self.H = int(T), int(H)
        self.depth = int(depth)
        if self.depth < 1:
            raise ValueError("HostPipeline: depth must be >= 1")
        self.x = [torch.empty((T, H), dtype=x_dtype, device=dev) for _ in range(self.depth)]
        self.y = [torch.empty((T, H), dtype=y_dtype, device=dev) for _ in range(self.depth)]
        self._computed = [None] * self.depth  # block done reading x[b] / writing y[b]
        self._copied_out = [None] * self.depth  # y[b] copied to the host
        self._n = 0
        self.device = dev

    def submit(self, x_host: torch.Tensor, y_host: torch.Tensor) -> torch.cuda.Event:
        if not (x_host.is_pinned() and y_host.is_pinned()):
            raise ValueError("HostPipeline.submit: x_host and y_host must be pinned host tensors")
        if tuple(x_host.shape) != (self.T, self.H) or tuple(y_host.shape) != (self.T, self.H):
            raise ValueError(f"HostPipeline.submit: expected [{self.T}, {self.H}] host tensors")
        b = self._n % self.depth
        self._n += 1
        compute = torch.cuda.current_stream(self.device)
        s_in, s_out = _host_streams(self.device)
        with torch.cuda.stream(s_in):
            if self._computed[b] is not None:
                s_in.wait_event(self._computed[b])
            self.x[b].copy_(x_host, non_blocking=True)
            copied_in = torch.cuda.Event()
            copied_in.record(s_in)
        compute.wait_event(copied_in)
        if self._copied_out[b] is not None:
            compute.wait_event(self._copied_out[b])
        self.block(self.x[b], out=self.y[b])
        computed = torch.cuda.Event()
        computed.record(compute)
        self._computed[b] = computed
        with torch.cuda.stream(s_out):
            s_out.wait_event(computed)
            y_host.copy_(self.y[b], non_blocking=True)
            done = torch.cuda.Event()
            done.record(s_out)
        self._copied_out[b] = done
        return done


_HOST_STREAMS: dict = {}


def _host_streams(dev):
    key = dev.index
    if key not in _HOST_STREAMS:
        _HOST_STREAMS[key] = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
    return _HOST_STREAMS[key]


class GraphedMoEFFN:
    """A :class:`MoEFFNBlock` call for a fixed token count captured once in a
    CUDA graph (the small, launch-bound decode steps).  ``x`` and ``y`` are the
    graph's static input and output buffers: copy tokens into ``x``, call
    :meth:`replay`, read ``y``.  The block's workspace is held for the life of
    this object."""

    def __init__(self, block: "MoEFFNBlock", T: int, device=None):
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.block = block
        self.x = torch.zeros((T, block.H), dtype=block.dtype, device=device)
        self.y = torch.empty((T, block.H), dtype=block.out_dtype, device=device)
        block._workspace(T, device)
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            block(self.x, out=self.y)  # warm-up outside capture (attributes, tensor maps)
        torch.cuda.current_stream(device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            block(self.x, out=self.y)
        torch.cuda.current_stream(device).wait_stream(side)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.y

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        if out is not None:
            out.copy_(self.y, non_blocking=True)
            return out
        return self.y


class GraphedHostMoEFFN:
    """A decode step from host memory to host memory as ONE CUDA graph: the
    copy of the tokens from the pinned host buffer ``x_host`` [T, H], the
    block and the copy of the result into the pinned host buffer ``y_host``
    [T, H] are captured together, so a step is a single graph launch.
    Write the tokens into ``x_host``, call :meth:`replay` (returns an event
    that completes when ``y_host`` holds the result), read ``y_host`` after
    the event.  ``x_host`` must not be modified before the event of the
    previous replay that reads it has completed."""

    def __init__(self, block: "MoEFFNBlock", T: int, device=None):
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.block = block
        self.x_host = torch.zeros((T, block.H), dtype=block.dtype).pin_memory()
        self.y_host = torch.zeros((T, block.H), dtype=block.out_dtype).pin_memory()
        self.x = torch.zeros((T, block.H), dtype=block.dtype, device=device)
        self.y = torch.empty((T, block.H), dtype=block.out_dtype, device=device)
        block._workspace(T, device)
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            block(self.x, out=self.y)  # warm-up outside capture (attributes, tensor maps)
        torch.cuda.current_stream(device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=side):
            self.x.copy_(self.x_host, non_blocking=True)
            block(self.x, out=self.y)
            self.y_host.copy_(self.y, non_blocking=True)
        torch.cuda.current_stream(device).wait_stream(side)

    def replay(self) -> torch.cuda.Event:
        self.graph.replay()
        done = torch.cuda.Event()
        done.record()
        return done


def read_device_error() -> int:
    """Return and clear the device error word of bounded in-kernel waits."""
    import ctypes

    v = ctypes.c_int32(0)
    _lib.check(_lib.load().frank_read_device_error(ctypes.byref(v), _stream()))
    return v.value


STAGE_NAMES = ("route", "permute", "gather", "gate_up_gemm", "down_gemm", "combine")


def launch_count() -> int:
    """Kernels launched by the library so far in this process."""
    return int(_lib.load().frank_launch_count())


def profile_stages(enable) -> None:
    """Record CUDA events around each stage of moe_ffn_block (measurement only).
    enable=2: graph-capture form (one event set, re-recorded by every replay)."""
    _lib.check(_lib.load().frank_profile_stages(2 if enable == 2 else int(bool(enable))))


def profile_read() -> dict:
    """Stage durations (ms) of the most recent profiled moe_ffn_block call."""
    import ctypes

    buf = (ctypes.c_float * len(STAGE_NAMES))()
    n = ctypes.c_int(0)
    _lib.check(_lib.load().frank_profile_read(buf, len(STAGE_NAMES), ctypes.byref(n)))
    return {name: float(buf[i]) for i, name in enumerate(STAGE_NAMES)}


def gather_rows(x: torch.Tensor, sorted_slots: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """xs[r] = x[sorted_slots[r] % T] for expert-sorted slots."""
    T, H = x.shape
    n = sorted_slots.numel()
    xs = out if out is not None else torch.empty((n, H), dtype=x.dtype, device=x.device)
    _lib.check(_lib.load().frank_gather_rows(_dt(x), _ptr(x), _ptr(sorted_slots), n, T, H, _ptr(xs), _stream()))
    return xs


def gather_weights(w: torch.Tensor, sorted_slots: torch.Tensor) -> torch.Tensor:
    out = torch.empty(sorted_slots.numel(), dtype=torch.float32, device=w.device)
    _lib.check(_lib.load().frank_gather_weights(_ptr(w), _ptr(sorted_slots), sorted_slots.numel(), _ptr(out),
                                                _stream()))
    return out


def expert_ffn(xs: torch.Tensor, w_rows: torch.Tensor, offsets: torch.Tensor, w_up_p: torch.Tensor,
               w_gate_p: torch.Tensor, w_down_p: torch.Tensor, out: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Grouped gate/up + swiglu + down x row weight over expert-sorted rows -> fp32 [rows, H]."""
    rows, H = xs.shape
    E, F, _ = w_up_p.shape
    lib = _lib.load()
    d = out if out is not None else torch.empty((rows, H), dtype=torch.float32, device=xs.device)
    need = lib.frank_expert_ffn_workspace_size(_dt(xs), rows, F)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=xs.device)
    _lib.check(lib.frank_expert_ffn(_dt(xs), _ptr(xs), _ptr(w_rows), _ptr(offsets), E, rows, H, F, _ptr(w_up_p),
                                    _ptr(w_gate_p), _ptr(w_down_p), _ptr(d), _ptr(workspace), workspace.numel(),
                                    _stream()))
    return d


def combine(d: torch.Tensor, slot_pos: torch.Tensor, T: int, k: int, out: torch.Tensor) -> torch.Tensor:
    """y[t] = sum_j d[slot_pos[j*T + t]] (j in order)."""
    H = d.shape[1]
    _lib.check(_lib.load().frank_combine(_ptr(d), _ptr(slot_pos), T, k, H, _dt(out), _ptr(out), _stream()))
    return out


def copy_row_segments(src: torch.Tensor, dst: torch.Tensor, src_start: torch.Tensor, dst_start: torch.Tensor,
                      seg_prefix: torch.Tensor, total_rows: int) -> None:
    """dst rows [dst_start[s], +len_s) = src rows [src_start[s], +len_s) (int64 device tables)."""
    row_bytes = src[0].numel() * src.element_size() if src.dim() > 1 else src.element_size()
    _lib.check(_lib.load().frank_copy_row_segments(_ptr(src), _ptr(dst), _ptr(src_start), _ptr(dst_start),
                                                   _ptr(seg_prefix), src_start.numel(), total_rows, row_bytes,
                                                   _stream()))
