"""ctypes binding to libavo_b200_attn.so, the sm_100a attention-forward library.

This is the host side of the candidate behind the AVO contract
``attention(q, k, v, causal)`` (reference: candidates/torch_sdpa_seed.py:6-7, the
loader avo/benchmark.py:406-418).  It restates the reference binding's argument
checks (candidates/cuda_mma_attention/attention.cpp:13-21: CUDA, contiguous,
equal shapes, rank 4; attention_kernel.cu:180-186: bf16, head_dim 128) and raises
``RuntimeError`` subclasses with the same meaning, then calls the C ABI declared in
include/avo_b200_attn.h on the tensors' current CUDA stream.

There is no fallback: if the library cannot be built or loaded, or the device is
not a B200, every call raises.  PyTorch is used only for device memory and streams.
"""

from __future__ import annotations

import ctypes
import importlib.util
import math
import sys
import threading
from pathlib import Path
from typing import Any

HERE = Path(__file__).resolve().parent

# Every function declared in include/avo_b200_attn.h, with (restype, argtypes).
_c_int, _c_ll, _c_float, _vp = ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_void_p
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "avo_b200_abi_version": (_c_int, []),
    "avo_b200_strerror": (ctypes.c_char_p, [_c_int]),
    "avo_b200_attn_fwd": (
        _c_int,
        [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _vp, _vp],
    ),
    "avo_b200_attn_fwd_block": (
        _c_int,
        [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
         _c_ll, _c_ll, _c_ll, _c_ll, _c_int, _c_float, _c_ll, _c_ll, _vp, _vp],
    ),
    "avo_b200_lse_merge": (
        _c_int,
        [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_ll, _c_ll, _c_ll, _c_ll, _vp],
    ),
    "avo_b200_acc_to_bf16": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_ll, _c_ll, _vp]),
    "avo_b200_watchdog_selftest": (_c_int, [_c_int, _vp, _vp]),
    "avo_b200_exp2_poly_eval": (_c_int, [_vp, _vp, _c_ll, _vp]),
    "avo_b200_attn_workspace_size": (_c_int, [ctypes.POINTER(ctypes.c_size_t)]),
    "avo_b200_attn_fwd_ws": (
        _c_int,
        [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _vp, ctypes.c_size_t,
         _vp, _vp],
    ),
    "avo_b200_schedule_units": (
        _c_int,
        [_c_int, _c_int, _c_int, _c_int, _c_ll, _c_ll, _c_int, _c_int, _vp, _vp, _c_int, _vp],
    ),
    "avo_b200_attn_fwd_split_noalloc": (
        _c_int,
        [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _vp, _vp],
    ),
}
ABI_VERSION = 1
HEAD_DIM = 128
STATUS_WATCHDOG = 1
STATUS_DRAIN = 2
NOALLOC_MAX_ROWS = 16384  # AVO_B200_NOALLOC_MAX_ROWS
ETOOBIG = 6
EREGS = 7


class B200AttentionError(RuntimeError):
    """A C-ABI call returned a non-zero code, or the device reported a watchdog abort."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
# The per-call entry avo_b200_attn_fwd_ws through the CPython binding in fast_call.c (bound
# to the address of the same function in the loaded library), or None where that binding
# was not built: the ctypes call is then used.
_fwd_ws_fast: Any = None
_status_words: dict[int, Any] = {}
_workspaces: dict[int, Any] = {}


def _build_module():
    name = "avo_b200_attention_build"
    module = sys.modules.get(name)
    if module is None:
        spec = importlib.util.spec_from_file_location(name, HERE / "build.py")
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
    return module


def library_path() -> Path:
    return _build_module().LIB_PATH


def load_library(*, build: bool = True) -> ctypes.CDLL:
    """Load (building first if missing or stale, when ``build``) the C-ABI library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        builder = _build_module()
        if build:
            builder.build()
        path = builder.LIB_PATH
        if not path.is_file():
            raise B200AttentionError(f"{path} is missing; run build.py")
        lib = ctypes.CDLL(str(path))
        for symbol, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, symbol)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.avo_b200_abi_version()
        if version != ABI_VERSION:
            raise B200AttentionError(f"ABI version {version} != expected {ABI_VERSION}")
        _bind_fast(builder, lib)
        _lib = lib
        return lib


def _bind_fast(builder, lib: ctypes.CDLL) -> None:
    global _fwd_ws_fast
    path = getattr(builder, "FAST_PATH", None)
    if path is None or not path.is_file():
        return
    spec = importlib.util.spec_from_file_location("_avo_b200_fast", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    module.bind(ctypes.cast(lib.avo_b200_attn_fwd_ws, ctypes.c_void_p).value)
    _fwd_ws_fast = module.fwd_ws


def strerror(code: int) -> str:
    return load_library().avo_b200_strerror(code).decode()


def _check(code: int, what: str) -> None:
    if code != 0:
        raise B200AttentionError(f"{what} failed: {strerror(code)} (code {code})")


def _torch():
    import torch

    return torch


def _stream_handle(device) -> int:
    return _torch().cuda.current_stream(device).cuda_stream


_raw_stream_getter: Any = None


def _raw_stream(index: int) -> int:
    """The current stream of device ``index`` as a cudaStream_t value.  torch's own raw
    getter costs ~0.1 us against ~3 us for building a Stream object; the public API is
    the fallback where the getter is absent."""
    global _raw_stream_getter
    if _raw_stream_getter is None:
        torch = _torch()
        getter = getattr(torch._C, "_cuda_getCurrentRawStream", None)
        _raw_stream_getter = getter if getter is not None else (
            lambda i: torch.cuda.current_stream(i).cuda_stream)
    return _raw_stream_getter(index)


_launch_states: dict[int, tuple[int, int, int]] = {}


def _launch_state(index: int) -> tuple[int, int, int]:
    """(workspace address, workspace bytes, status word address) of device ``index``,
    looked up once per device (both buffers live for the life of the process)."""
    state = _launch_states.get(index)
    if state is None:
        ws = workspace(index)
        state = (ws.data_ptr(), ws.numel(), status_word(index).data_ptr())
        _launch_states[index] = state
    return state


def status_word(device) -> Any:
    """Per-device int32 word that kernels OR their watchdog bits into."""
    torch = _torch()
    index = torch.device(device).index
    if index is None:
        index = torch.cuda.current_device()
    word = _status_words.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=f"cuda:{index}")
        _status_words[index] = word
    return word


def workspace(device) -> Any:
    """Per-device scratch for split work items (uint8, zero-filled once at allocation; the
    kernel leaves it zeroed after every launch that completes).  Allocated by torch's
    caching allocator on first use and kept for the life of the process."""
    torch = _torch()
    index = torch.device(device).index
    if index is None:
        index = torch.cuda.current_device()
    ws = _workspaces.get(index)
    if ws is None:
        size = ctypes.c_size_t(0)
        with torch.cuda.device(index):
            _check(load_library().avo_b200_attn_workspace_size(ctypes.byref(size)),
                   "avo_b200_attn_workspace_size")
        ws = torch.zeros(int(size.value), dtype=torch.uint8, device=f"cuda:{index}")
        _workspaces[index] = ws
    return ws


def check_status(device, *, reset: bool = True) -> int:
    """Synchronize ``device``'s status word; raise if a kernel reported an abort.  After an
    abort the device's split-piece workspace is zeroed again (its flags may be stale)."""
    word = status_word(device)
    value = int(word.item())
    if reset and value:
        word.zero_()
        index = word.device.index
        if index in _workspaces:
            _workspaces[index].zero_()
    if value & (STATUS_WATCHDOG | STATUS_DRAIN):
        raise B200AttentionError(
            f"device watchdog fired (status {value}): a kernel pipeline wait timed out; "
            "outputs of that launch are invalid"
        )
    return value


def _validate(q, k, v) -> None:
    torch = _torch()
    # The common, valid case in one pass of cheap attribute reads; any failure falls
    # through to the checks below, which raise what the reference binding would.
    if q.is_cuda and k.is_cuda and v.is_cuda and q.is_contiguous() and k.is_contiguous() and v.is_contiguous():
        shape = q.shape
        bf16 = torch.bfloat16
        if (shape == k.shape and shape == v.shape and len(shape) == 4 and q.dtype is bf16 and k.dtype is bf16
                and v.dtype is bf16 and shape[3] == HEAD_DIM and q.get_device() == k.get_device() == v.get_device()):
            return
    # Same checks, same order, as the reference binding (attention.cpp:13-21).
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous")
    if q.shape != k.shape:
        raise RuntimeError("q and k must have the same shape")
    if q.shape != v.shape:
        raise RuntimeError("q and v must have the same shape")
    if q.dim() != 4:
        raise RuntimeError("q, k, and v must have shape (batch, heads, seq, dim)")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"{name} must be bf16")
    if q.shape[3] != HEAD_DIM:
        raise RuntimeError("head_dim must be 128")
    if not (q.device == k.device == v.device):
        raise RuntimeError("q, k, and v must be on the same device")


def default_scale(head_dim: int = HEAD_DIM) -> float:
    return 1.0 / math.sqrt(head_dim)


def attention_forward(q, k, v, causal: bool, *, softmax_scale: float | None = None,
                      need_lse: bool = True, out=None, lse=None, split: bool = True):
    """O (bf16, like q) and LSE (fp32 [B, H, S], natural log, or None) of SDPA.

    With ``split`` (the default) the call goes through ``avo_b200_attn_fwd_ws`` with the
    device's workspace, which lets the kernel cut work items between CTAs where whole
    items would leave SMs idle; ``split=False`` calls ``avo_b200_attn_fwd``, whole items
    only."""
    torch = _torch()
    _validate(q, k, v)
    batch, heads, seq, head_dim = q.shape
    if out is None:
        out = torch.empty_like(q)
    if need_lse and lse is None:
        lse = torch.empty((batch, heads, seq), dtype=torch.float32, device=q.device)
    if not need_lse:
        lse = None
    scale = default_scale(head_dim) if softmax_scale is None else float(softmax_scale)
    lib = _lib if _lib is not None else load_library()
    # The call costs a few microseconds of host time, which is what small problems are
    # bound by: per-device state is cached, the raw current stream is read directly, and
    # the device is switched only when q is not on the current one.
    index = q.get_device()
    ws_ptr, ws_bytes, status_ptr = _launch_state(index)
    lse_ptr = lse.data_ptr() if lse is not None else None

    def call() -> int:
        if split:
            return (_fwd_ws_fast or lib.avo_b200_attn_fwd_ws)(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse_ptr,
                batch, heads, seq, head_dim, 1 if causal else 0, scale, ws_ptr, ws_bytes,
                status_ptr, _raw_stream(index))
        return lib.avo_b200_attn_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse_ptr,
            batch, heads, seq, head_dim, 1 if causal else 0, scale, status_ptr, _raw_stream(index))

    if index == torch.cuda.current_device():
        code = call()
    else:
        with torch.cuda.device(index):
            code = call()
    _check(code, "avo_b200_attn_fwd_ws" if split else "avo_b200_attn_fwd")
    return out, lse


def attention_forward_noalloc(q, k, v, causal: bool, *, n_splits: int = 2, softmax_scale: float | None = None,
                              need_lse: bool = True, out=None, lse=None):
    """attention_forward through avo_b200_attn_fwd_split_noalloc: the key/value range in
    n_splits blocks merged by log-sum-exp in the library's static scratch (no device
    allocation by the library; B*H*S <= NOALLOC_MAX_ROWS).  Calls must not overlap in
    time on one device: the scratch is shared."""
    torch = _torch()
    _validate(q, k, v)
    batch, heads, seq, head_dim = (int(x) for x in q.shape)
    if out is None:
        out = torch.empty_like(q)
    if need_lse and lse is None:
        lse = torch.empty((batch, heads, seq), dtype=torch.float32, device=q.device)
    if not need_lse:
        lse = None
    scale = default_scale(head_dim) if softmax_scale is None else float(softmax_scale)
    lib = load_library()
    with torch.cuda.device(q.device):
        code = lib.avo_b200_attn_fwd_split_noalloc(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            lse.data_ptr() if lse is not None else None,
            batch, heads, seq, head_dim, 1 if causal else 0, scale, int(n_splits),
            status_word(q.device).data_ptr(), _stream_handle(q.device),
        )
    _check(code, "avo_b200_attn_fwd_split_noalloc")
    return out, lse


def attention_block(q, k, v, out, lse, *, causal: bool, q_pos0: int, kv_pos0: int,
                    softmax_scale: float | None = None) -> None:
    """Block attention on [num_bh, rows, 128] views (rows contiguous, any head stride).

    ``q``/``out`` are [num_bh, seq_q, 128] bf16, ``k``/``v`` [num_bh, seq_kv, 128] bf16,
    ``lse`` fp32 [num_bh, seq_q] (row-contiguous); positions drive the causal mask.
    """
    torch = _torch()
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.dim() != 3 or t.shape[2] != HEAD_DIM or t.stride(2) != 1 or t.stride(1) != HEAD_DIM:
            raise RuntimeError(f"{name} must be [num_bh, rows, 128] with contiguous rows")
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"{name} must be bf16")
    if k.stride(0) != v.stride(0) or k.shape != v.shape:
        raise RuntimeError("k and v must share shape and head stride")
    if lse is not None and (lse.dim() != 2 or lse.stride(1) != 1 or lse.dtype != torch.float32):
        raise RuntimeError("lse must be fp32 [num_bh, seq_q] with contiguous rows")
    num_bh, seq_q, _ = (int(x) for x in q.shape)
    seq_kv = int(k.shape[1])
    scale = default_scale() if softmax_scale is None else float(softmax_scale)
    lib = load_library()
    with torch.cuda.device(q.device):
        code = lib.avo_b200_attn_fwd_block(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            lse.data_ptr() if lse is not None else None,
            num_bh, seq_q, seq_kv, HEAD_DIM,
            q.stride(0), k.stride(0), out.stride(0), lse.stride(0) if lse is not None else seq_q,
            1 if causal else 0, scale, int(q_pos0), int(kv_pos0),
            status_word(q.device).data_ptr(), _stream_handle(q.device),
        )
    _check(code, "avo_b200_attn_fwd_block")


def _rows_view(t, name, dtype):
    if t.dim() != 3 or t.shape[2] != HEAD_DIM or t.stride(2) != 1 or t.stride(1) != HEAD_DIM:
        raise RuntimeError(f"{name} must be [num_bh, rows, 128] with contiguous rows")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}")


def _lse_view(t, name):
    torch = _torch()
    if t.dim() != 2 or t.stride(1) != 1 or t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be fp32 [num_bh, rows] with contiguous rows")


def lse_merge(acc_o, acc_lse, part_o, part_lse) -> None:
    """Fold one partial (bf16 O, fp32 LSE) into fp32 accumulators by log-sum-exp."""
    torch = _torch()
    _rows_view(acc_o, "acc_o", torch.float32)
    _rows_view(part_o, "part_o", torch.bfloat16)
    _lse_view(acc_lse, "acc_lse")
    _lse_view(part_lse, "part_lse")
    if acc_o.shape != part_o.shape or tuple(acc_lse.shape) != tuple(acc_o.shape[:2]) or \
            tuple(part_lse.shape) != tuple(acc_o.shape[:2]):
        raise RuntimeError("lse_merge shapes disagree")
    num_bh, rows, head_dim = (int(x) for x in acc_o.shape)
    lib = load_library()
    with torch.cuda.device(acc_o.device):
        code = lib.avo_b200_lse_merge(
            acc_o.data_ptr(), acc_lse.data_ptr(), part_o.data_ptr(), part_lse.data_ptr(),
            num_bh, rows, head_dim, acc_o.stride(0), acc_lse.stride(0), part_o.stride(0),
            part_lse.stride(0), _stream_handle(acc_o.device),
        )
    _check(code, "avo_b200_lse_merge")


def acc_to_bf16(acc_o, out) -> None:
    """out (bf16) = acc_o (fp32), both [num_bh, rows, 128] with contiguous rows."""
    torch = _torch()
    _rows_view(acc_o, "acc_o", torch.float32)
    _rows_view(out, "out", torch.bfloat16)
    if acc_o.shape != out.shape:
        raise RuntimeError("acc_to_bf16 shapes disagree")
    num_bh, rows, head_dim = (int(x) for x in acc_o.shape)
    lib = load_library()
    with torch.cuda.device(acc_o.device):
        code = lib.avo_b200_acc_to_bf16(
            acc_o.data_ptr(), out.data_ptr(), num_bh, rows, head_dim, acc_o.stride(0),
            out.stride(0), _stream_handle(acc_o.device),
        )
    _check(code, "avo_b200_acc_to_bf16")


def watchdog_selftest(device, timeout_us: int = 20000) -> int:
    """Run the never-completing-wait kernel; returns the status bits it reported."""
    torch = _torch()
    word = torch.zeros(1, dtype=torch.int32, device=device)
    lib = load_library()
    with torch.cuda.device(word.device):
        code = lib.avo_b200_watchdog_selftest(int(timeout_us), word.data_ptr(),
                                              _stream_handle(word.device))
    _check(code, "avo_b200_watchdog_selftest")
    return int(word.item())


def exp2_poly_eval(x):
    """The kernel's FMA-pipe 2^x on a CUDA fp32 tensor (diagnostic; inputs in [-125, 127])."""
    torch = _torch()
    if not x.is_cuda or x.dtype != torch.float32 or not x.is_contiguous():
        raise RuntimeError("x must be a contiguous CUDA fp32 tensor")
    y = torch.empty_like(x)
    lib = load_library()
    with torch.cuda.device(x.device):
        code = lib.avo_b200_exp2_poly_eval(x.data_ptr(), y.data_ptr(), x.numel(), _stream_handle(x.device))
    _check(code, "avo_b200_exp2_poly_eval")
    return y


def schedule_units(num_bh: int, seq_q: int, seq_kv: int, causal: bool, *, sm_count: int = 148,
                   split: bool = True, q_pos0: int = 0, kv_pos0: int = 0, max_units: int = 512):
    """The kernel's work plan, enumerated on the host (no GPU needed): returns
    (mode, grid, run_min, wave_items, units) where units[c] lists CTA c's units as
    (bh, q0, t0, t1, kind, seg, cont_lo, cont_hi) in processing order."""
    import numpy as np

    lib = load_library()
    plan = (ctypes.c_int * 4)()
    code = lib.avo_b200_schedule_units(num_bh, seq_q, seq_kv, 1 if causal else 0, q_pos0, kv_pos0, sm_count,
                                       1 if split else 0, plan, None, max_units, None)
    _check(code, "avo_b200_schedule_units")
    grid = plan[1]
    units = np.zeros((max(grid, 1), max_units, 8), dtype=np.int32)
    counts = np.zeros(max(grid, 1), dtype=np.int32)
    code = lib.avo_b200_schedule_units(num_bh, seq_q, seq_kv, 1 if causal else 0, q_pos0, kv_pos0, sm_count,
                                       1 if split else 0, plan, units.ctypes.data, max_units, counts.ctypes.data)
    _check(code, "avo_b200_schedule_units")
    if (counts > max_units).any():
        raise ValueError(f"more than {max_units} units per CTA")
    return plan[0], grid, plan[2], plan[3], [units[c, :counts[c]].tolist() for c in range(grid)]
