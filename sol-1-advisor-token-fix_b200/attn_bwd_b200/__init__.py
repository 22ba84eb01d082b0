"""B200 (sm_100a) GQA attention backward behind the reference's entry point.

``custom_kernel(data) -> (grad_attn_scores, grad_value_states)`` keeps the
signature of the reference's ``attn_bwd/starting_point.py:27-70`` (and of
``attn_bwd/submission.py``), so it drops in wherever the reference harness calls
it (``eval_modal_attn_bwd.py:273,339,381``; ``append.py:29-33``).  The work runs
in two hand-written sm_100a kernels reached through the C-ABI of
``include/attn_bwd_b200.h``; inputs must be CUDA tensors and there is no CPU
fallback.
"""
import torch

from . import _lib
from ._lib import AttnBwdError

NUM_ATTENTION_HEADS = 80
NUM_KEY_VALUE_HEADS = 8
NUM_GROUPS = NUM_ATTENTION_HEADS // NUM_KEY_VALUE_HEADS
HEAD_DIM = 128

__all__ = ["custom_kernel", "attn_bwd", "attn_bwd_shard", "attn_bwd_host", "ds_shard", "dv_shard", "run",
           "AttnBwdError", "poll_error", "release", "options", "attn_bwd_from_mask", "NUM_ATTENTION_HEADS", "NUM_KEY_VALUE_HEADS",
           "HEAD_DIM"]


def _ptr(t):
    return ctypes_void(t.data_ptr())


def ctypes_void(x):
    import ctypes
    return ctypes.c_void_p(x)


def _stream():
    return ctypes_void(torch.cuda.current_stream().cuda_stream)


def _prep(t, name, dtype, shape, flexible=False):
    """Checks one input the way the reference's ops would see it and returns a
    contiguous, 16-byte-aligned view (a copy only if the caller's is not)."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a torch.Tensor, got {type(t).__name__}")
    if t.device.type != "cuda":
        raise ValueError(f"{name}: tensor must be on a CUDA device (no CPU path), got {t.device}")
    if t.dtype != dtype:
        raise TypeError(f"{name}: expected dtype {dtype}, got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        n = 1
        for x in shape:
            n *= x
        if flexible and t.numel() == n and t.is_contiguous():
            t = t.view(shape)
        else:
            raise ValueError(f"{name}: expected shape {tuple(shape)}, got {tuple(t.shape)}")
    if not t.is_contiguous() or t.data_ptr() % 16:
        t = t.contiguous() if t.is_contiguous() is False else t.clone()
    return t


def _shapes(grad_attn_output, value_states):
    if grad_attn_output.dim() != 4 or value_states.dim() != 4:
        raise ValueError("grad_attn_output and value_states must be 4-D")
    bs, sq, h, d = grad_attn_output.shape
    skv = value_states.shape[2]
    if h != NUM_ATTENTION_HEADS or d != HEAD_DIM:
        raise ValueError(f"grad_attn_output must be [bs, seq_q, {NUM_ATTENTION_HEADS}, {HEAD_DIM}], "
                         f"got {tuple(grad_attn_output.shape)}")
    return bs, sq, skv


def _check_inputs(data, u0=None, u1=None):
    (dO, P, Pd, V, M, p) = data
    bs, sq, skv = _shapes(dO, V)
    if u0 is None:
        u0, u1 = 0, bs * NUM_KEY_VALUE_HEADS
    if not (0 <= u0 <= u1 <= bs * NUM_KEY_VALUE_HEADS):
        raise ValueError(f"unit range [{u0},{u1}) outside [0,{bs * NUM_KEY_VALUE_HEADS}]")
    nh = (u1 - u0) * NUM_GROUPS
    full = (u0 == 0 and u1 == bs * NUM_KEY_VALUE_HEADS)
    sshape = (bs, NUM_ATTENTION_HEADS, sq, skv) if full else (nh, sq, skv)
    dO = _prep(dO, "grad_attn_output", torch.bfloat16, (bs, sq, NUM_ATTENTION_HEADS, HEAD_DIM))
    V = _prep(V, "value_states", torch.bfloat16, (bs, NUM_KEY_VALUE_HEADS, skv, HEAD_DIM))
    if P is not None:
        P = _prep(P, "attn_weights", torch.bfloat16, sshape, flexible=True)
    if Pd is not None:
        Pd = _prep(Pd, "attn_weights_dropped", torch.bfloat16, sshape, flexible=True)
    if M is not None:
        M = _prep(M, "dropout_mask", torch.bool, sshape, flexible=True)
    devs = {t.device for t in (dO, P, Pd, V, M) if t is not None}
    if len(devs) != 1:
        raise ValueError(f"all tensors must be on one CUDA device, got {devs}")
    return dO, P, Pd, V, M, float(p), bs, sq, skv, u0, u1


def attn_bwd_shard(data, unit_begin, unit_end, out=None):
    """Attention backward for units u = b*8 + kv_head in [unit_begin, unit_end).

    ``data`` is the reference tuple, except that attn_weights,
    attn_weights_dropped and dropout_mask hold only the shard's heads
    ([(unit_end-unit_begin)*10, seq_q, seq_kv]).  Returns (dS_shard [nh, sq, skv],
    dV_shard [units, skv, 128]).
    """
    dO, P, Pd, V, M, p, bs, sq, skv, u0, u1 = _check_inputs(data, unit_begin, unit_end)
    nh = (u1 - u0) * NUM_GROUPS
    with torch.cuda.device(dO.device):
        if out is None:
            dS = torch.empty((nh, sq, skv), dtype=torch.bfloat16, device=dO.device)
            dV = torch.empty((u1 - u0, skv, HEAD_DIM), dtype=torch.bfloat16, device=dO.device)
        else:
            dS, dV = out
        _lib.call("attn_bwd_b200_shard", _ptr(dO), _ptr(P), _ptr(Pd), _ptr(V), _ptr(M), p,
                  bs, sq, skv, u0, u1, _ptr(dS), _ptr(dV), _stream())
    return dS, dV


def attn_bwd_host(data, unit_begin=None, unit_end=None, device=None, work=None, out=None, chunks=0,
                  synchronize=True):
    """Attention backward for inputs and outputs in HOST memory, with the host<->device
    copies pipelined against the kernels (C-ABI ``attn_bwd_b200_host_shard``).

    ``data`` is the reference tuple of CPU tensors (contiguous, exact dtypes; pinned memory
    lets the copies overlap).  With a unit range, attn_weights, attn_weights_dropped and
    dropout_mask hold only the shard's heads, as in :func:`attn_bwd_shard`.  ``work`` is an
    optional tuple of 7 device tensors (dO, P, P_drop, V, mask, dS, dV) of the same sizes,
    reused across calls; otherwise they are allocated on ``device`` (default: current).
    ``out`` optionally supplies the host (dS, dV) tensors.  Returns (dS, dV) on the host;
    with ``synchronize=False`` they are valid only once the current stream has finished.
    """
    dO, P, Pd, V, M, p = data
    for t, name in ((dO, "grad_attn_output"), (V, "value_states")):
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu":
            raise TypeError(f"{name} must be a CPU tensor for attn_bwd_host")
    bs, sq, skv = _shapes(dO, V)
    u0 = 0 if unit_begin is None else unit_begin
    u1 = bs * NUM_KEY_VALUE_HEADS if unit_end is None else unit_end
    if not (0 <= u0 <= u1 <= bs * NUM_KEY_VALUE_HEADS):
        raise ValueError(f"unit range [{u0},{u1}) outside [0,{bs * NUM_KEY_VALUE_HEADS}]")
    nh = (u1 - u0) * NUM_GROUPS
    full = unit_begin is None and unit_end is None
    sshape = (bs, NUM_ATTENTION_HEADS, sq, skv) if full else (nh, sq, skv)
    vshape = (bs, NUM_KEY_VALUE_HEADS, skv, HEAD_DIM) if full else (u1 - u0, skv, HEAD_DIM)
    spec = [(dO, "grad_attn_output", torch.bfloat16, (bs, sq, NUM_ATTENTION_HEADS, HEAD_DIM)),
            (P, "attn_weights", torch.bfloat16, sshape), (Pd, "attn_weights_dropped", torch.bfloat16, sshape),
            (V, "value_states", torch.bfloat16, (bs, NUM_KEY_VALUE_HEADS, skv, HEAD_DIM)),
            (M, "dropout_mask", torch.bool, sshape)]
    for t, name, dt, shape in spec:
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu":
            raise TypeError(f"{name} must be a CPU tensor for attn_bwd_host")
        if t.dtype != dt or tuple(t.shape) != tuple(shape) or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dt} tensor of shape {tuple(shape)}, "
                             f"got {t.dtype} {tuple(t.shape)}")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if work is None:
        work = tuple(torch.empty(tuple(t.shape), dtype=t.dtype, device=dev) for t in (dO, P, Pd, V, M)) + (
            torch.empty(sshape, dtype=torch.bfloat16, device=dev),
            torch.empty(vshape, dtype=torch.bfloat16, device=dev))
    if len(work) != 7:
        raise ValueError("work must hold 7 device tensors (dO, P, P_drop, V, mask, dS, dV)")
    sizes = [dO, P, Pd, V, M, P, None]
    for w, ref in zip(work, sizes):
        want = (ref.numel() * ref.element_size()) if ref is not None else (u1 - u0) * skv * HEAD_DIM * 2
        if not w.is_cuda or not w.is_contiguous() or w.numel() * w.element_size() != want:
            raise ValueError("work tensors must be contiguous CUDA tensors with the inputs' and outputs' sizes")
    if out is None:
        pin = torch.cuda.is_available()
        dS_h = torch.empty(sshape, dtype=torch.bfloat16, pin_memory=pin)
        dV_h = torch.empty(vshape, dtype=torch.bfloat16, pin_memory=pin)
    else:
        dS_h, dV_h = out
    with torch.cuda.device(work[0].device):
        _lib.call("attn_bwd_b200_host_shard", *(_ptr(t) for t in (dO, P, Pd, V, M)), float(p), bs, sq, skv, u0, u1,
                  _ptr(dS_h), _ptr(dV_h), *(_ptr(w) for w in work), int(chunks), _stream())
        if synchronize:
            torch.cuda.current_stream().synchronize()
            # the stream is idle: a kernel wait that gave up would otherwise go unnoticed
            rc = _lib.load().attn_bwd_b200_poll_error()
            if rc:
                raise AttnBwdError("attn_bwd_b200_host_shard", _lib.EKERNEL if rc > 0xFF else rc)
    return dS_h, dV_h


_BF16 = torch.bfloat16


def _fast_ok(dO, P, Pd, V, M):
    """True when the inputs need no conversion: CUDA tensors of the right dtypes and
    shapes, contiguous, 16-byte aligned, on one device (checked cheaply, per call)."""
    try:
        if not (dO.is_cuda and dO.dtype is _BF16 and P.dtype is _BF16 and Pd.dtype is _BF16 and
                V.dtype is _BF16 and M.dtype is torch.bool):
            return False
        bs, sq, h, d = dO.shape
        skv = V.shape[2]
        if (h != NUM_ATTENTION_HEADS or d != HEAD_DIM or
                V.shape != (bs, NUM_KEY_VALUE_HEADS, skv, HEAD_DIM) or
                P.shape != (bs, NUM_ATTENTION_HEADS, sq, skv) or Pd.shape != P.shape or M.shape != P.shape):
            return False
        dev = dO.device
        for t in (P, Pd, V, M):
            if t.device != dev:
                return False
        for t in (dO, P, Pd, V, M):
            if not t.is_contiguous() or t.data_ptr() & 15:
                return False
        return True
    except (AttributeError, ValueError, TypeError):
        return False


try:
    _raw_stream = torch._C._cuda_getCurrentRawStream   # int handle of the current stream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def _stream_handle(device_index):
    if _raw_stream is not None:
        return _raw_stream(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def _load_torch_fast():
    """The C++ host binding (csrc/torch_fast.cpp), or None when it is not built or when
    ATTN_BWD_B200_LIB selects another build of the library (the binding links the
    in-tree one)."""
    import os
    if os.environ.get("ATTN_BWD_B200_LIB") or os.environ.get("ATTN_BWD_NO_TORCH_BINDING"):
        return None
    try:
        from . import _torch_fast
    except ImportError:
        return None
    return _torch_fast.fast


_torch_fast_fn = _load_torch_fast()


def attn_bwd(data, out=None):
    """Full call; returns fresh (dS [bs,80,sq,skv], dV [bs,8,skv,128]) bf16 tensors
    unless ``out`` supplies preallocated ones."""
    dO, P, Pd, V, M, p = data
    if out is None and _torch_fast_fn is not None and isinstance(dO, torch.Tensor):
        try:
            r = _torch_fast_fn(dO, P, Pd, V, M, float(p))
        except TypeError:   # not tensors: the general path reports it
            r = None
        if r is not None:
            if isinstance(r, int):
                raise AttnBwdError("attn_bwd_b200", r)
            return r
    if out is None and _fast_ok(dO, P, Pd, V, M):
        idx = dO.device.index
        if idx != torch.cuda.current_device():
            with torch.cuda.device(idx):
                return attn_bwd(data)
        dS = torch.empty_like(P)
        dV = torch.empty_like(V)
        bs, sq = dO.shape[0], dO.shape[1]
        rc = _lib.fast_fn()(dO.data_ptr(), P.data_ptr(), Pd.data_ptr(), V.data_ptr(), M.data_ptr(), float(p),
                            bs, sq, V.shape[2], dS.data_ptr(), dV.data_ptr(), _stream_handle(idx))
        if rc:
            raise AttnBwdError("attn_bwd_b200", rc)
        return dS, dV
    dO, P, Pd, V, M, p, bs, sq, skv, u0, u1 = _check_inputs(data)
    with torch.cuda.device(dO.device):
        if out is None:
            dS = torch.empty((bs, NUM_ATTENTION_HEADS, sq, skv), dtype=torch.bfloat16, device=dO.device)
            dV = torch.empty((bs, NUM_KEY_VALUE_HEADS, skv, HEAD_DIM), dtype=torch.bfloat16, device=dO.device)
        else:
            dS, dV = out
        _lib.call("attn_bwd_b200", _ptr(dO), _ptr(P), _ptr(Pd), _ptr(V), _ptr(M), p,
                  bs, sq, skv, _ptr(dS), _ptr(dV), _stream())
    return dS, dV


def custom_kernel(data):
    """Drop-in for the reference's ``custom_kernel`` (starting_point.py:27-70).

    data = (grad_attn_output [bs,sq,80,128] bf16, attn_weights [bs,80,sq,skv] bf16,
            attn_weights_dropped [bs,80,sq,skv] bf16, value_states [bs,8,skv,128] bf16,
            dropout_mask [bs,80,sq,skv] bool, attention_dropout float)
    returns (grad_attn_scores [bs,80,sq,skv] bf16, grad_value_states [bs,8,skv,128] bf16),
    ordered on ``torch.cuda.current_stream()``.
    """
    if not isinstance(data, (tuple, list)) or len(data) != 6:
        raise ValueError("custom_kernel expects the 6-tuple (grad_attn_output, attn_weights, "
                         "attn_weights_dropped, value_states, dropout_mask, attention_dropout)")
    return attn_bwd(tuple(data))


@torch.no_grad()
def run(grad_attn_output, attn_weights, attn_weights_dropped, value_states, dropout_mask,
        attention_dropout):
    """Keyword wrapper with the signature of the reference harness's ``run``
    (append.py:29-33)."""
    return custom_kernel((grad_attn_output, attn_weights, attn_weights_dropped, value_states,
                          dropout_mask, attention_dropout))


def attn_bwd_from_mask(data, unit_begin=None, unit_end=None, out=None):
    """The full call WITHOUT attn_weights_dropped (C-ABI ``attn_bwd_b200_shard_from_mask``):
    the dV kernel forms P_drop = bf16(attn_weights * dropout_mask / (1 - p)) itself.

    Only valid when the caller's P_drop is that product, which is how the reference's
    inputs are made (eval_modal_attn_bwd.py:159-161); for any other P_drop use
    :func:`custom_kernel`.  ``data`` is the reference tuple with attn_weights_dropped
    ignored (it may be None).  Needs 0 <= p < 1 and seq_kv % 16 == 0.  With a unit range the
    shard conventions of :func:`attn_bwd_shard` apply and (dS_shard, dV_shard) come back;
    without, the reference's output shapes."""
    dO, P, _, V, M, p = data
    full = unit_begin is None and unit_end is None
    dO, P, _, V, M, p, bs, sq, skv, u0, u1 = _check_inputs((dO, P, None, V, M, p), unit_begin, unit_end)
    nh = (u1 - u0) * NUM_GROUPS
    with torch.cuda.device(dO.device):
        if out is None:
            if full:
                dS = torch.empty((bs, NUM_ATTENTION_HEADS, sq, skv), dtype=torch.bfloat16, device=dO.device)
                dV = torch.empty((bs, NUM_KEY_VALUE_HEADS, skv, HEAD_DIM), dtype=torch.bfloat16, device=dO.device)
            else:
                dS = torch.empty((nh, sq, skv), dtype=torch.bfloat16, device=dO.device)
                dV = torch.empty((u1 - u0, skv, HEAD_DIM), dtype=torch.bfloat16, device=dO.device)
        else:
            dS, dV = out
        _lib.call("attn_bwd_b200_shard_from_mask", _ptr(dO), _ptr(P), _ptr(V), _ptr(M), p, bs, sq, skv, u0, u1,
                  _ptr(dS), _ptr(dV), _stream())
    return dS, dV


def ds_shard(dO, P, V, M, p, unit_begin, unit_end, out=None):
    """dS kernel alone (same shard conventions as :func:`attn_bwd_shard`)."""
    dO, P, _, V, M, p, bs, sq, skv, u0, u1 = _check_inputs((dO, P, None, V, M, p), unit_begin, unit_end)
    nh = (u1 - u0) * NUM_GROUPS
    with torch.cuda.device(dO.device):
        dS = out if out is not None else torch.empty((nh, sq, skv), dtype=torch.bfloat16, device=dO.device)
        _lib.call("attn_bwd_b200_ds_shard", _ptr(dO), _ptr(P), _ptr(V), _ptr(M), p, bs, sq, skv,
                  u0, u1, _ptr(dS), _stream())
    return dS


def dv_shard(dO, Pd, V, unit_begin, unit_end, out=None):
    """dV kernel alone (same shard conventions as :func:`attn_bwd_shard`)."""
    dO, _, Pd, V, _, _, bs, sq, skv, u0, u1 = _check_inputs((dO, None, Pd, V, None, 0.0), unit_begin, unit_end)
    with torch.cuda.device(dO.device):
        dV = out if out is not None else torch.empty((u1 - u0, skv, HEAD_DIM), dtype=torch.bfloat16,
                                                     device=dO.device)
        _lib.call("attn_bwd_b200_dv_shard", _ptr(dO), _ptr(Pd), bs, sq, skv, u0, u1, _ptr(dV), _stream())
    return dV


def poll_error():
    """Synchronise and return (and clear) the code of a kernel wait that gave up; 0 if none."""
    return _lib.load().attn_bwd_b200_poll_error()


def release():
    """Synchronise the current device and free the library's lazily created streams,
    events and cached launch graphs on it (later calls re-create them)."""
    _lib.call("attn_bwd_b200_release")


class options:
    """Context manager forcing measurement / test options of the library for its body,
    e.g. ``with options(ds_mode=3): ...`` (names and values: ATTN_BWD_OPT_* in
    include/attn_bwd_b200.h).  Process-wide; the previous values are restored on exit."""

    def __init__(self, **opts):
        for k in opts:
            if k not in _lib.OPTIONS:
                raise ValueError(f"unknown option {k!r}; known: {sorted(_lib.OPTIONS)}")
        self.opts = opts
        self.saved = {}

    def __enter__(self):
        for k, v in self.opts.items():
            self.saved[k] = _lib.get_option(k)
            _lib.set_option(k, v)
        return self

    def __exit__(self, *exc):
        for k, v in self.saved.items():
            _lib.set_option(k, v)
        return False
