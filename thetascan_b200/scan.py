"""The ``b200`` scan backend: drop-in for the reference chunk scan.

Mirrors ``thetascan._core.ops.scan_chunk`` (src/thetascan/_core/ops/
scan_chunk.py:86, 246-358): same function names, argument meaning, output
dtype and errors, computed by the sm_100a kernels behind the C ABI
(``ts_b200_scan_fwd`` / ``ts_b200_scan_bwd``).  ``chunk`` is validated like the
reference's but does not change the result: the kernels tile the sequence in
128-token tiles internally, and the chunked algebra is exact for any tile.

Supported: bf16 streams on the tensor cores and float32 streams on the CUDA
cores (f32 FMAs: the float32 tolerance of the reference is out of reach of
bf16 or tf32 operands), on a CUDA device, with the plain causal sum
(``None``), static per-head log-retentions (``[H]``) and per-token
log-retention streams (``[B,H,T,1]``, on the float32 CUDA-core kernels for
either stream dtype: per-tile cumulative log phases, one closing factor per
tile), up to four retentions per call, ``Dk`` and ``Dv`` up to 256 within
the CTA budgets (float32: ``Dk = 128`` with ``Dv <= 248``, ``Dk = 256`` with
``Dv <= 123``).  Mixed stream dtypes raise ``NotImplementedError``; a
non-CUDA tensor raises ``RuntimeError``.  Nothing falls back to a CPU
implementation.

A stream's weights are the exact products ``exp(L_t - L_i)`` of its
cumulative log-retention.  The reference clamps the intra-chunk exponent at
zero (scan_chunk.py:150-153), which only acts on positive entries (growth)
and then depends on its chunk width; for entries <= 0 the two agree.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

DEFAULT_CHUNK = 512


def _strides3(x: torch.Tensor):
    s = x.stride()
    if s[3] != 1:
        raise ValueError("b200 scan: the innermost dimension must be contiguous")
    return _lib.c_int64_3(s[0], s[1], s[2])


def _ptr(x):
    return ctypes.c_void_p(0 if x is None else x.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _is_stream(r):
    return r is not None and r.ndim == 4


def _flat_retentions(retentions):
    """Static ``[H]`` and stream ``[B,H,T,1]`` retentions as contiguous f32
    (a stream flattens to the kernels' ``[B,H,T]`` layout)."""
    return [None if r is None else r.detach().reshape(-1).to(torch.float32).contiguous() for r in retentions]


def _build_args(q, k, v, las, outs, append_unit, workspace=None, stale=None, streams=None):
    B, H, T, Dk = q.shape
    a = _lib.ScanArgs()
    a.batch, a.heads, a.tokens, a.dk = B, H, T, Dk
    n_unit = int(append_unit)   # False/True/2: constant columns after v
    a.dv = v.shape[-1] + n_unit
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.q_strides, a.k_strides, a.v_strides = _strides3(q), _strides3(k), _strides3(v)
    a.v_append_unit = n_unit
    a.n_retentions = len(las)
    for i, la in enumerate(las):
        stream = bool(streams and streams[i])
        a.log_alpha[i] = None if (la is None or stream) else la.data_ptr()
        a.log_alpha_stream[i] = la.data_ptr() if (la is not None and stream) else None
        a.stale[i] = 1 if (stale and stale[i]) else 0
        if outs is not None:
            a.out[i] = outs[i].data_ptr()
    a.out_dtype = _lib.TS_DTYPE_BF16 if (outs is not None and outs[0].dtype == torch.bfloat16) else _lib.TS_DTYPE_F32
    a.f32_streams = 1 if q.dtype == torch.float32 else 0
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    return a


def _workspace(lib, fn, args, device):
    nbytes = fn(ctypes.byref(args))
    if nbytes == 0:
        _lib.check(_lib.last_error()[0] or _lib.TS_ERR_VALUE)
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _scan_fwd_impl(q, k, v, retentions, append_unit, stale, round_streams):
    """Body of the ``thetascan_b200::scan_views_fwd`` op: f32 reads of every
    retention, stacked ``[R,B,H,T,Dv(+unit)]``, and the workspace that holds
    the carried chunk states for the backward."""
    lib = _lib.load()
    q, k, v = _operand_streams(q, k, v, retentions, round_streams)
    las = _flat_retentions(retentions)
    streams = [_is_stream(r) for r in retentions]
    B, H, T, _ = q.shape
    dv = v.shape[-1] + append_unit
    # The kernels write f32 reads; the backward's log-retention term uses
    # them unrounded, and the caller casts them to the stream dtype.
    outs_all = torch.empty(len(las), B, H, T, dv, dtype=torch.float32, device=q.device)
    args = _build_args(q, k, v, las, list(outs_all.unbind(0)), append_unit, stale=stale if any(stale) else None,
                       streams=streams)
    ws = _workspace(lib, lib.ts_b200_scan_workspace_bytes, args, q.device)
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.ts_b200_scan_fwd(ctypes.byref(args), _stream()))
    return outs_all, ws


def _operand_streams(q, k, v, retentions, round_streams):
    """The q, k, v the kernels read: per-token retention streams run on the
    float32 CUDA-core kernels (bf16 streams are widened, exactly), otherwise
    ``round_streams`` rounds float32 streams to bf16 for the tensor cores."""
    if any(_is_stream(r) for r in retentions):
        return tuple(x.to(torch.float32) for x in (q, k, v))
    if round_streams:
        return tuple(x.to(torch.bfloat16).contiguous() for x in (q, k, v))
    return q, k, v


def _scan_bwd_impl(douts, q, k, v, retentions, outs_all, ws, append_unit, stale, round_streams):
    """Body of the ``thetascan_b200::scan_views_bwd`` op: f32 gradients of q,
    k, v (without the unit columns), ``[R,H]`` static log-retention gradients
    and ``[S,B,H,T]`` gradients of the S per-token retention streams."""
    lib = _lib.load()
    q, k, v = _operand_streams(q, k, v, retentions, round_streams)
    las = _flat_retentions(retentions)
    streams = [_is_stream(r) for r in retentions]
    n = len(las)
    B, H, T, Dk = q.shape
    dv_width = outs_all.shape[-1]
    # bf16 streams take bf16 read gradients; f32 streams keep them f32
    gdt = torch.float32 if q.dtype == torch.float32 else torch.bfloat16
    dgrads = [douts[i].to(gdt).contiguous() for i in range(n)]
    args = _build_args(q, k, v, las, list(outs_all.unbind(0)), append_unit, ws, stale=stale if any(stale) else None,
                       streams=streams)
    g = _lib.ScanGradArgs()
    dq = torch.empty(B, H, T, Dk, dtype=torch.float32, device=q.device)
    dk = torch.empty_like(dq)
    dvv = torch.empty(B, H, T, dv_width, dtype=torch.float32, device=q.device)
    dla = torch.zeros(n, H, dtype=torch.float32, device=q.device)
    dstream = torch.empty(sum(streams), B, H, T, dtype=torch.float32, device=q.device)
    s_index = 0
    for i in range(n):
        g.dout[i] = dgrads[i].data_ptr()
        if streams[i]:
            g.dlog_alpha_stream[i] = dstream[s_index].data_ptr()
            s_index += 1
        else:
            g.dlog_alpha[i] = None if las[i] is None else dla[i].data_ptr()
    g.dq, g.dk, g.dv = dq.data_ptr(), dk.data_ptr(), dvv.data_ptr()
    g.grad_dtype = _lib.TS_DTYPE_F32
    gws = _workspace(lib, lib.ts_b200_scan_bwd_workspace_bytes, args, q.device)
    g.workspace, g.workspace_bytes = gws.data_ptr(), gws.numel()
    _lib.check(lib.ts_b200_scan_bwd(ctypes.byref(args), ctypes.byref(g), _stream()))
    if append_unit:
        dvv = dvv[..., :v.shape[-1]].contiguous()
    return dq, dk, dvv, dla, dstream


def _scan_views_op(q, k, v, retentions, append_unit, stale, round_streams):
    """The multi-view scan as the ``thetascan_b200::scan_views_fwd`` custom op
    (autograd and fake implementation registered in :mod:`thetascan_b200.ops`);
    returns the f32 reads of every retention."""
    from . import ops  # noqa: F401  (registers the operators)
    outs_all, _ = torch.ops.thetascan_b200.scan_views_fwd(
        q, k, v, [r for r in retentions if r is not None], [r is not None for r in retentions], int(append_unit),
        [bool(x) for x in stale], bool(round_streams))
    return outs_all.unbind(0)


def scan_views_f32(q, k, v, append_unit, stale, retentions):
    """The multi-view scan of float32 q, k, v on bf16 streams: the inputs are
    rounded to bf16 inside (what the tensor-core kernels read), the reads are
    f32, and the gradients return in float32 as the kernels write them, with
    no bf16 round trip on the way back.  Used by callers whose per-token math
    around the scan is float32 (the GN family)."""
    flags = [bool(x) for x in stale] if stale is not None else [False] * len(retentions)
    return tuple(_scan_views_op(q, k, v, retentions, append_unit, flags, True))


def _check_inputs(q, k, v, retentions, chunk):
    if chunk < 1:
        raise ValueError("chunk backend: chunk must be >= 1")
    for x in (q, k, v):
        if not x.is_cuda:
            raise RuntimeError("b200 backend requires CUDA tensors")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in (torch.bfloat16, torch.float32):
        raise NotImplementedError(
            "b200 backend: q, k and v must all be bf16 (tensor cores) or all float32 (CUDA cores), "
            f"got {q.dtype}, {k.dtype}, {v.dtype}")
    B, H, T = q.shape[:3]
    for r in retentions:
        if r is None:
            continue
        if r.ndim == 4:
            if r.shape[-1] != 1:
                raise NotImplementedError("chunk backend: scalar decay only (v1)")
            if tuple(r.shape[:3]) != (B, H, T):
                raise ValueError(
                    f"b200 scan: a retention stream must be [B,H,T,1], got {tuple(r.shape)} for q {tuple(q.shape)}")
            if not r.is_cuda:
                raise RuntimeError("b200 backend requires CUDA tensors")
            continue
        if r.numel() != H:
            raise ValueError(
                "chunk backend: a static retention needs one entry per head, "
                f"got {tuple(r.shape)} for q {tuple(q.shape)}")


def linattn_views(q, k, v, retentions, chunk: int = DEFAULT_CHUNK, *, append_unit: bool = False, stale=None):
    """Scan one stream set through several retentions (scan_chunk.py:246-339).

    ``append_unit=True`` treats the payload as ``[v | 1]`` without
    materialising it (the key-mass read of engine.py:430); the outputs then have
    ``Dv + 1`` columns, the last being the retention-weighted score mass.
    ``stale`` (one flag per retention) reads a static retention's stale view,
    weights ``1 - alpha^(t-i)``: the reference's ``FadeStale`` difference
    ``S_sum - S_fast`` (interface.py:251-279), formed inside the kernels.
    """
    if not retentions:
        return ()
    _check_inputs(q, k, v, retentions, chunk)
    stale = tuple(bool(x) for x in stale) if stale is not None else (False,) * len(retentions)
    if len(stale) != len(retentions):
        raise ValueError("b200 scan: one stale flag per retention")
    for r, st in zip(retentions, stale):
        if st and r is None:
            raise ValueError("b200 scan: a stale view needs a retention")
    streams = any(_is_stream(r) for r in retentions)
    if any(stale) and (q.dtype == torch.float32 or streams):
        # float32 kernels: the stale view as the reference forms it, S_sum -
        # S_fast (FadeStale.scan_terms, interface.py:268-273); the difference
        # loses nothing the float32 tolerance would see
        wide = tuple(x.to(torch.float32) for x in (q, k, v))
        reads = linattn_views(*wide, tuple(retentions) + (None,), chunk, append_unit=append_unit)
        return tuple((reads[-1] - o if st else o).to(q.dtype) for o, st in zip(reads[:-1], stale))
    outs = []
    # The kernels take at most four retentions per call; longer tuples are split.
    for start in range(0, len(retentions), _lib.MAX_RETENTIONS):
        group = tuple(retentions[start:start + _lib.MAX_RETENTIONS])
        flags = stale[start:start + _lib.MAX_RETENTIONS]
        outs.extend(o.to(q.dtype) for o in _scan_views_op(q, k, v, group, int(append_unit), flags, False))
    return tuple(outs)


def linattn(q, k, v, decay=None, chunk: int = DEFAULT_CHUNK, log_alpha=None):
    """One-view scan (scan_chunk.py:342-358); ``log_alpha`` takes precedence."""
    retention = log_alpha if log_alpha is not None else decay
    return linattn_views(q, k, v, (retention,), chunk)[0]


def _stream_fwd_impl(q, k, v, retentions, append_unit, state):
    """Body of ``thetascan_b200::scan_views_stream_fwd``: the forward scan of
    one segment with boundary states (``ts_scan_args.init_state`` /
    ``final_state``)."""
    lib = _lib.load()
    las = [None if r is None else r.detach().reshape(-1).to(torch.float32).contiguous() for r in retentions]
    B, H, T, Dk = q.shape
    dv = v.shape[-1] + append_unit
    if state is not None:
        if tuple(state.shape) != (B, H, len(las), Dk, dv) or state.dtype != torch.float32:
            raise ValueError(f"b200 streaming scan: state must be f32 [{B},{H},{len(las)},{Dk},{dv}]")
        state = state.contiguous()
    outs_all = torch.empty(len(las), B, H, T, dv, dtype=torch.float32, device=q.device)
    new_state = torch.empty(B, H, len(las), Dk, dv, dtype=torch.float32, device=q.device)
    args = _build_args(q, k, v, las, list(outs_all.unbind(0)), append_unit)
    ws = _workspace(lib, lib.ts_b200_scan_workspace_bytes, args, q.device)
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    args.init_state = None if state is None else state.data_ptr()
    args.final_state = new_state.data_ptr()
    _lib.check(lib.ts_b200_scan_fwd(ctypes.byref(args), _stream()))
    return outs_all, new_state, ws


def _stream_bwd_impl(douts, dstate, q, k, v, retentions, outs_all, ws, append_unit, state):
    """Body of ``thetascan_b200::scan_views_stream_bwd``: the backward of one
    segment from the gradients of its reads and of its leaving state
    (``ts_scan_grad_args.dfinal_state``), with the gradient of the entering
    state (``dinit_state``)."""
    lib = _lib.load()
    las = [None if r is None else r.detach().reshape(-1).to(torch.float32).contiguous() for r in retentions]
    n = len(las)
    B, H, T, Dk = q.shape
    dv_width = outs_all.shape[-1]
    dgrads = [douts[i].to(torch.bfloat16).contiguous() for i in range(n)]
    args = _build_args(q, k, v, las, list(outs_all.unbind(0)), append_unit, ws)
    if state is not None:
        state = state.contiguous()
        args.init_state = state.data_ptr()
    g = _lib.ScanGradArgs()
    dq = torch.empty(B, H, T, Dk, dtype=torch.float32, device=q.device)
    dk = torch.empty_like(dq)
    dvv = torch.empty(B, H, T, dv_width, dtype=torch.float32, device=q.device)
    dla = torch.zeros(n, H, dtype=torch.float32, device=q.device)
    dstate = dstate.to(torch.float32).contiguous()
    dinit = torch.empty_like(state) if state is not None else None
    for i in range(n):
        g.dout[i] = dgrads[i].data_ptr()
        g.dlog_alpha[i] = None if las[i] is None else dla[i].data_ptr()
    g.dq, g.dk, g.dv = dq.data_ptr(), dk.data_ptr(), dvv.data_ptr()
    g.grad_dtype = _lib.TS_DTYPE_F32
    g.dfinal_state = dstate.data_ptr()
    g.dinit_state = None if dinit is None else dinit.data_ptr()
    gws = _workspace(lib, lib.ts_b200_scan_bwd_workspace_bytes, args, q.device)
    g.workspace, g.workspace_bytes = gws.data_ptr(), gws.numel()
    _lib.check(lib.ts_b200_scan_bwd(ctypes.byref(args), ctypes.byref(g), _stream()))
    if append_unit:
        dvv = dvv[..., :v.shape[-1]].contiguous()
    return dq, dk, dvv, dla, (q.new_empty(0, dtype=torch.float32) if dinit is None else dinit)


def linattn_views_stream(q, k, v, retentions, state=None, *, append_unit: bool = False):
    """Streaming form of :func:`linattn_views`: scan this segment of the
    sequence continuing from ``state`` and return ``(outputs, new_state)``,
    differentiable in the streams, the retentions and ``state``.

    ``state`` is what the previous segment returned (``None`` for the start
    of the sequence): f32 ``[B,H,R,Dk,Dv]`` with ``R = len(retentions)`` and
    ``Dv`` the payload width (``+1`` with ``append_unit``), the carried chunk
    state of every retention -- the persistent fast state of a decoder.
    Scanning a sequence segment by segment gives the outputs of one call over
    the whole sequence (to rounding), for segments of any lengths, and the
    backward through the chain of segments gives the one call's gradients
    (the state's gradient flows from each segment into the one before)."""
    if not retentions:
        return (), state
    _check_inputs(q, k, v, retentions, DEFAULT_CHUNK)
    if q.dtype == torch.float32:
        raise NotImplementedError("b200 streaming scan: bf16 streams only")
    if any(_is_stream(r) for r in retentions):
        raise NotImplementedError("b200 streaming scan: static retentions only (per-token streams take linattn_views)")
    if len(retentions) > _lib.MAX_RETENTIONS:
        raise NotImplementedError(f"b200 streaming scan: at most {_lib.MAX_RETENTIONS} retentions per call")
    from . import ops  # noqa: F401  (registers the operators)
    outs_all, new_state, _ = torch.ops.thetascan_b200.scan_views_stream_fwd(
        q, k, v, [r for r in retentions if r is not None], [r is not None for r in retentions], int(append_unit),
        state)
    return tuple(o.to(q.dtype) for o in outs_all.unbind(0)), new_state
