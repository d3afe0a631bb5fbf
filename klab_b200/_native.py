"""ctypes binding of libklab_b200.so (include/klab_b200.h).

The reference drives its native layer through ctypes too (kernel_lab.py:120-130,
cuda_module.py:149-158). There is no fallback: importing an operator module on
a machine without the built library raises immediately, and every projection
runs the sm_100a kernels of this library.
"""

from __future__ import annotations

import ctypes as ct
import os
import threading
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"
# KLAB_B200_LIBRARY selects another build of the same library (e.g. one compiled
# with different ring depth or warp count); the default is the in-tree build.
LIB_PATH = Path(os.environ.get("KLAB_B200_LIBRARY", LIB_DIR / "libklab_b200.so"))
PREFETCH_CUBIN = LIB_DIR / "prefetch_kernels.cubin"

# include/klab_b200.h constants
DT_BF16, DT_F16, DT_F32 = 0, 1, 2
W_BF16, W_F16, W_F32, W_CBF16, W_I8_ROW, W_I8_G64, W_FP4_G32H, W_FP4_G16E, W_LF32, W_FP28 = range(10)
FP4_E4M3_G16, FP4_F16_G32 = 0, 1
L2_HINT, L2_HINT_LAST, L2_LOAD, L2_BULK = 0, 1, 2, 3
OPT_PDL, OPT_SPLIT, OPT_GENERIC, OPT_CTAS_PER_SM, OPT_TENSOR, OPT_PROLOGUE, OPT_MAX_TILE = 0, 1, 2, 3, 4, 5, 6
E_DRIVER, E_NO_CONTEXT, E_INVALID = -1000, -1001, -1002
E_SHAPE, E_ALIGN, E_UNSUPPORTED, E_DEVICE, E_SCRATCH = -2001, -2002, -2003, -2004, -2005

_P = ct.c_void_p
_I = ct.c_int
_SZ = ct.c_size_t
_SIGNATURES = {
    "klab_gemv": (_I, [_I, _I, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P]),
    "klab_gemv_multi": (_I, [_I, _I, _P, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _SZ, _P]),
    "klab_gemv_multi_gather": (_I, [_I, _I, _P, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "klab_ipc_malloc": (_I, [_SZ, ct.POINTER(_P), _P]),
    "klab_ipc_open": (_I, [_P, ct.POINTER(_P)]),
    "klab_ipc_close": (_I, [_P]),
    "klab_ipc_free": (_I, [_P]),
    "klab_step_begin": (_I, [_P, _P]),
    "klab_chain_create": (_I, [_P, _I, _P, ct.POINTER(_P)]),
    "klab_chain_launch": (_I, [_P, _P]),
    "klab_chain_destroy": (_I, [_P]),
    "klab_chain_info": (_I, [_P, ct.POINTER(_I), ct.POINTER(_I)]),
    "klab_chain_trace": (_I, [_P, _P, _SZ]),
    "klab_wait_flags": (_I, [_P, _I, _I, _P, _P]),
    "klab_raw_linear": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P]),
    "klab_raw_linear_noalloc": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "klab_coded_linear": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P]),
    "klab_half_linear": (_I, [_P, _P, _I, _P, _I, _I, _I, _P, _SZ, _P]),
    "klab_f32_linear": (_I, [_P, _P, _P, _I, _I, _I, _P, _SZ, _P]),
    "klab_residual_rmsnorm": (_I, [_P, _P, _P, _P, _I, _I, ct.c_float, _P]),
    "klab_add_rmsnorm": (_I, [_P, _P, _P, _P, _P, _I, _I, ct.c_float, _P]),
    "klab_silu_mul": (_I, [_P, _P, _I, _I, _P]),
    "klab_decode_attention": (_I, [_P, _P, _P, _P, _P, _P, _P, ct.c_longlong, _P, _P, _I, _I, _I, _I, ct.c_float,
                                    _P]),
    "klab_add_rmsnorm_linear": (_I, [_P, _P, _P, ct.c_float, _P, _P, _P, _I, _I, _I, _P, _SZ, _P]),
    "klab_silu_mul_linear": (_I, [_P, _P, _P, _I, _I, _I, _P, _SZ, _P]),
    "klab_int8_linear": (_I, [_P, _I, _P, _P, _I, _P, _I, _I, _I, _I, _P, _SZ, _P]),
    "klab_fp4_linear": (_I, [_P, _I, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P, _SZ, _P]),
    "klab_lossless_f32_linear": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _SZ, _P]),
    "klab_fp28_linear": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _SZ, _P]),
    "klab_lossless_f32_unpack": (_I, [_P, _P, _P, _P, ct.c_longlong, _P]),
    "klab_fp28_unpack": (_I, [_P, _P, _P, ct.c_longlong, _P]),
    "klab_gemv_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "klab_plan_create": (_I, [_I, _I, _I, _I, _I, _I, ct.POINTER(_P)]),
    "klab_plan_launch": (_I, [_P, _P, _P, _P, _P, _P, _P, _P]),
    "klab_plan_info": (_I, [_P, ct.c_char_p, _SZ]),
    "klab_plan_destroy": (_I, [_P]),
    "klab_cbf16_unpack": (_I, [_P, _P, _P, _I, _I, _P]),
    "klab_int8_dequantize": (_I, [_P, _P, _I, _P, _I, _I, _P]),
    "klab_fp4_dequantize": (_I, [_P, _P, _I, _P, _P, _I, _I, _P]),
    "klab_cbf16_pack_host": (_I, [_P, _I, _I, _P, _P, _SZ, ct.POINTER(_SZ)]),
    "klab_cbf16_unpack_host": (_I, [_P, _SZ, _P, _I, _I, _P]),
    "klab_l2_prefetch": (_I, [_P, ct.c_longlong, _I, _I, _I, _I, _P, _P]),
    "klab_set_option": (_I, [_I, _I]),
    "klab_get_option": (_I, [_I]),
    "klab_device_status": (_I, [_I]),
    "klab_error_string": (ct.c_char_p, [_I]),
    "klab_version": (_I, []),
    "lab_load_ptx": (_I, [ct.c_char_p, ct.POINTER(_P)]),
    "lab_load_file": (_I, [ct.c_char_p, ct.POINTER(_P)]),
    "lab_get_kernel": (_I, [_P, ct.c_char_p, ct.POINTER(_P)]),
    "lab_launch": (_I, [_P, ct.c_uint, ct.c_uint, ct.c_uint, _P, ct.POINTER(_P)]),
    "lab_launch_ex": (_I, [_P, ct.c_uint, ct.c_uint, ct.c_uint, ct.c_uint, ct.c_uint, _P, ct.POINTER(_P)]),
    "lab_unload": (_I, [_P]),
    "lab_error_string": (ct.c_char_p, [_I]),
}
EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


class KlabError(RuntimeError):
    """A native call failed; .code is the klab / CUDA error code."""

    def __init__(self, code, what):
        self.code = code
        super().__init__(f"{what} failed ({code}): {error_string(code)}")


def lib():
    """The loaded library. Raises when it has not been built (no fallback)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m klab_b200.build` "
                                       "(klab_b200 has no CPU or framework fallback)")
                handle = ct.CDLL(str(LIB_PATH))
                for name, (restype, argtypes) in _SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype, fn.argtypes = restype, argtypes
                _lib = handle
    return _lib


def error_string(code: int) -> str:
    text = lib().klab_error_string(int(code))
    return text.decode() if text else "unknown error"


def check(code: int, what: str) -> None:
    if code:
        raise KlabError(code, what)


def ptr(tensor) -> int:
    return tensor.data_ptr()


def current_stream(device):
    import torch

    return torch.cuda.current_stream(device)


def record(stream, *tensors):
    """ctypes launches bypass the caching allocator's stream bookkeeping
    (kernel_lab.py:183-186); tell it which stream used each tensor."""
    import torch

    if torch.cuda.is_current_stream_capturing():
        return
    for t in tensors:
        if t is not None:
            t.record_stream(stream)


class _Workspaces:
    """Per (device, stream) split-K workspace: zero-filled once, grown outside
    graph capture, then reused by every launch on that stream (launches leave
    it zeroed)."""

    def __init__(self):
        self._buffers = {}
        self._lock = threading.Lock()

    def get(self, device_index: int, stream, need: int):
        import torch

        if need <= 0:
            return None
        key = (device_index, int(stream.cuda_stream))
        with self._lock:
            buf = self._buffers.get(key)
            if buf is not None and buf.numel() >= need:
                return buf
            if torch.cuda.is_current_stream_capturing():
                return buf if buf is not None and buf.numel() >= need else None
            size = max(need, 1 << 20)
            buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", device_index))
            self._buffers[key] = buf
            return buf


WORKSPACES = _Workspaces()


def workspace_for(wfmt: int, m: int, n: int, k: int, device_index: int, stream):
    need = lib().klab_gemv_workspace_bytes(wfmt, m, n, k)
    buf = WORKSPACES.get(device_index, stream, int(need))
    if buf is None:
        return None, 0
    return buf.data_ptr(), buf.numel()


def set_option(option: int, value: int) -> None:
    check(lib().klab_set_option(option, value), "klab_set_option")


def get_option(option: int) -> int:
    return lib().klab_get_option(option)


def device_status(clear: bool = True) -> int:
    """The current device's status word (0: no kernel gave up a bounded wait)."""
    value = lib().klab_device_status(1 if clear else 0)
    if value < 0 or value > 16:
        raise KlabError(value, "klab_device_status")
    return value


def gemv(wfmt, xdt, x, w, aux, gscale, out, out_dt, m, n, k, *, ldx=None, ldo=None, workspace=True):
    """Launch one projection on torch's current stream of x's device."""
    import torch

    device = x.device
    stream = torch.cuda.current_stream(device)
    ws_ptr, ws_bytes = (workspace_for(wfmt, m, n, k, device.index, stream) if workspace else (None, 0))
    with torch.cuda.device(device):
        rc = lib().klab_gemv(wfmt, xdt, x.data_ptr(), k if ldx is None else ldx, w.data_ptr(),
                             None if aux is None else aux.data_ptr(),
                             None if gscale is None else gscale.data_ptr(), out.data_ptr(),
                             n if ldo is None else ldo, out_dt, m, n, k, ws_ptr, ws_bytes, stream.cuda_stream)
    check(rc, "klab_gemv")
    record(stream, x, w, aux, gscale, out)
    return out


MAX_PEERS = 8


class Gather(ct.Structure):
    """klab_gather_t: an output gather fused into a projection (peer stores plus
    a completion flag), and/or a bounded wait for the peers' flags before x is read."""

    _fields_ = [("npeers", _I), ("rank", _I), ("seg", _I), ("peer_out", _P * MAX_PEERS),
                ("peer_flags", _P * MAX_PEERS), ("signal_slot", _I), ("wait_flags", _P), ("wait_slot", _I),
                ("epoch", _P), ("done", _P)]


def make_gather(npeers, rank, epoch, *, seg=-1, peer_out=(), peer_flags=(), signal_slot=-1, wait_flags=None,
                wait_slot=-1, done=None):
    """A Gather from raw device addresses (ints)."""
    g = Gather()
    g.npeers, g.rank, g.seg = npeers, rank, seg
    for q, a in enumerate(peer_out):
        g.peer_out[q] = a
    for q, a in enumerate(peer_flags):
        g.peer_flags[q] = a
    g.signal_slot, g.wait_flags, g.wait_slot = signal_slot, wait_flags, wait_slot
    g.epoch, g.done = epoch, done
    return g


class ChainStage(ct.Structure):
    """klab_chain_stage_t: one stage of the persistent chain kernel."""

    _fields_ = [("x", _P), ("k", _I), ("nseg", _I), ("w", _P * 8), ("out", _P * 8), ("n", _I * 8),
                ("gather_seg", _I), ("peer_out", _P * MAX_PEERS), ("x_stage", _I)]


class ChainSync(ct.Structure):
    """klab_chain_sync_t: ranks, step counter and the step output of a chain."""

    _fields_ = [("npeers", _I), ("rank", _I), ("epoch", _P), ("final_in", _P), ("final_out", _P)]


def chain_create(stages, sync) -> int:
    """Upload a persistent chain plan; stages is a list of ChainStage."""
    arr = (ChainStage * len(stages))(*stages)
    plan = ct.c_void_p()
    check(lib().klab_chain_create(arr, len(stages), ct.byref(sync), ct.byref(plan)), "klab_chain_create")
    return plan.value


def chain_launch(plan: int, stream) -> None:
    check(lib().klab_chain_launch(plan, stream.cuda_stream), "klab_chain_launch")


def chain_info(plan: int):
    """(CTAs per launch, trace slots per (stage, CTA)) of a chain plan."""
    grid, slots = ct.c_int(), ct.c_int()
    check(lib().klab_chain_info(plan, ct.byref(grid), ct.byref(slots)), "klab_chain_info")
    return grid.value, slots.value


def chain_trace(plan: int, buffer) -> None:
    """Record a timeline into `buffer` (int64 CUDA tensor, or None to stop)."""
    if buffer is None:
        check(lib().klab_chain_trace(plan, None, 0), "klab_chain_trace")
    else:
        check(lib().klab_chain_trace(plan, buffer.data_ptr(), buffer.numel() * buffer.element_size()),
              "klab_chain_trace")


def chain_destroy(plan: int) -> None:
    check(lib().klab_chain_destroy(plan), "klab_chain_destroy")


def plan_create(wfmt, xdt, out_dt, m, n, k) -> int:
    """A prepared launch for one case on the current device (klab_plan_create)."""
    plan = ct.c_void_p()
    check(lib().klab_plan_create(wfmt, xdt, out_dt, m, n, k, ct.byref(plan)), "klab_plan_create")
    return plan.value


def plan_info(plan: int) -> str:
    buf = ct.create_string_buffer(1024)
    check(lib().klab_plan_info(plan, buf, len(buf)), "klab_plan_info")
    return buf.value.decode()


def plan_launch(plan: int, x, w, aux, aux2, gscale, out, stream) -> None:
    ptr_or_none = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    check(lib().klab_plan_launch(plan, x.data_ptr(), w.data_ptr(), ptr_or_none(aux), ptr_or_none(aux2),
                                 ptr_or_none(gscale), out.data_ptr(), stream.cuda_stream), "klab_plan_launch")


def plan_destroy(plan: int) -> None:
    check(lib().klab_plan_destroy(plan), "klab_plan_destroy")


def ipc_malloc(nbytes: int):
    """Zero-filled device memory on the current device and its 64-byte IPC handle."""
    p = ct.c_void_p()
    handle = ct.create_string_buffer(64)
    check(lib().klab_ipc_malloc(nbytes, ct.byref(p), handle), "klab_ipc_malloc")
    return p.value, handle.raw


def ipc_open(handle: bytes) -> int:
    p = ct.c_void_p()
    buf = ct.create_string_buffer(bytes(handle), 64)
    check(lib().klab_ipc_open(buf, ct.byref(p)), "klab_ipc_open")
    return p.value


def ipc_close(address: int) -> None:
    check(lib().klab_ipc_close(address), "klab_ipc_close")


def ipc_free(address: int) -> None:
    check(lib().klab_ipc_free(address), "klab_ipc_free")


def step_begin(epoch, stream) -> None:
    check(lib().klab_step_begin(epoch.data_ptr(), stream.cuda_stream), "klab_step_begin")


def wait_flags(flags: int, slot: int, npeers: int, epoch, stream) -> None:
    check(lib().klab_wait_flags(flags, slot, npeers, epoch.data_ptr(), stream.cuda_stream), "klab_wait_flags")


def gemv_multi(wfmt, xdt, x, segments, gscale, out_dt, m, k, *, ldx=None, workspace=True, gather=None):
    """One launch over several projections sharing x: segments is a list of
    (w, aux, out_view, ldo, n_rows); out_view points at the first output element.
    gather (a Gather) fuses an output push to the peers and/or a wait for them."""
    import torch

    nseg = len(segments)
    device = x.device
    stream = torch.cuda.current_stream(device)
    total = sum(seg[4] for seg in segments)
    ws_ptr, ws_bytes = (workspace_for(wfmt, m, total, k, device.index, stream) if workspace else (None, 0))
    wp = (ct.c_void_p * nseg)(*[seg[0].data_ptr() for seg in segments])
    ap = (ct.c_void_p * nseg)(*[(seg[1].data_ptr() if seg[1] is not None else None) for seg in segments])
    op = (ct.c_void_p * nseg)(*[seg[2].data_ptr() for seg in segments])
    ldo = (ct.c_int * nseg)(*[seg[3] for seg in segments])
    ns = (ct.c_int * nseg)(*[seg[4] for seg in segments])
    with torch.cuda.device(device):
        if gather is None:
            rc = lib().klab_gemv_multi(wfmt, xdt, x.data_ptr(), k if ldx is None else ldx, nseg, wp, ap,
                                       None if gscale is None else gscale.data_ptr(), op, ldo, ns, out_dt, m, k,
                                       ws_ptr, ws_bytes, stream.cuda_stream)
        else:
            rc = lib().klab_gemv_multi_gather(wfmt, xdt, x.data_ptr(), k if ldx is None else ldx, nseg, wp, ap,
                                              None if gscale is None else gscale.data_ptr(), op, ldo, ns, out_dt,
                                              m, k, ct.byref(gather), ws_ptr, ws_bytes, stream.cuda_stream)
    check(rc, "klab_gemv_multi")
    record(stream, x, *[t for seg in segments for t in (seg[0], seg[1], seg[2])])
