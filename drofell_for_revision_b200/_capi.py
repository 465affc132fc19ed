"""ctypes binding of the C ABI declared in include/drofell_w4a16.h.

The library is built in-tree (``python -m drofell_for_revision_b200.build``). There
is no fallback: if the library is missing or CUDA is unavailable, every entry point
raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdrofell_w4a16.so")

W4A16_OK = 0
W4A16_ERR_INVALID = 1
W4A16_ERR_CUDA = 2
W4A16_ERR_UNSUPPORTED = 3
W4A16_ERR_WORKSPACE = 4

DTYPE_FP16 = 0
DTYPE_BF16 = 1

PATH_AUTO = 0
PATH_GEMV = 1
PATH_TC = 2
PATH_TC_EXACT = 3

KERN_GEMV = 1
KERN_EXACT = 3
KERN_GEMV_MMA = 4

EXPORTED = (
    "w4a16_create", "w4a16_destroy", "w4a16_dequant", "w4a16_workspace_size", "w4a16_gemm",
    "w4a16_plan", "w4a16_info", "w4a16_device_error", "w4a16_last_error", "w4a16_version",
    "w4a16_gemm_static",
    "w4a16_comm_create", "w4a16_comm_destroy", "w4a16_comm_flags", "w4a16_comm_set_peer_flags",
    "w4a16_ipc_export", "w4a16_ipc_open", "w4a16_ipc_close", "w4a16_gemm_gather",
    "w4a16_plan_shape", "w4a16_create_ex", "w4a16_gemm_t", "w4a16_workspace_size_t",
    "w4a16_rms_norm", "w4a16_silu_mul", "w4a16_mlp_forward", "w4a16_mlp_workspace_size", "w4a16_qkv_forward",
    "w4a16_qkv_workspace_size",
)
CREATE_NO_REPACK = 1
IPC_HANDLE_BYTES = 72

_lib = None
_lock = threading.Lock()


class W4A16Error(RuntimeError):
    """A failure reported by the C ABI (carries the W4A16_ERR_* code)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[w4a16 error {code}] {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"W4A16 CUDA library not built ({LIB_PATH}); run `python -m drofell_for_revision_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        P, I, S = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        IP = ctypes.POINTER(ctypes.c_int)
        L.w4a16_create.argtypes = [P, P, P, P, I, I, I, I, P, ctypes.POINTER(P)]
        L.w4a16_create.restype = I
        L.w4a16_create_ex.argtypes = [P, P, P, P, I, I, I, I, I, P, ctypes.POINTER(P)]
        L.w4a16_create_ex.restype = I
        L.w4a16_gemm_t.argtypes = [P, P, I, P, I, P, S, P]
        L.w4a16_gemm_t.restype = I
        L.w4a16_workspace_size_t.argtypes = [P, I, I]
        L.w4a16_workspace_size_t.restype = S
        F = ctypes.c_float
        L.w4a16_rms_norm.argtypes = [P, P, F, I, I, P, I, P]
        L.w4a16_rms_norm.restype = I
        L.w4a16_silu_mul.argtypes = [P, P, I, I, P, I, P]
        L.w4a16_silu_mul.restype = I
        L.w4a16_mlp_forward.argtypes = [P, P, P, P, F, P, I, P, P, P, P, I, P, S, P]
        L.w4a16_mlp_forward.restype = I
        L.w4a16_mlp_workspace_size.argtypes = [P, P, P, I, I]
        L.w4a16_mlp_workspace_size.restype = S
        L.w4a16_qkv_forward.argtypes = [P, P, P, P, F, P, I, P, P, P, P, I, P, S, P]
        L.w4a16_qkv_forward.restype = I
        L.w4a16_qkv_workspace_size.argtypes = [P, P, P, I, I]
        L.w4a16_qkv_workspace_size.restype = S
        L.w4a16_destroy.argtypes = [P]
        L.w4a16_destroy.restype = I
        L.w4a16_dequant.argtypes = [P, P, I, P]
        L.w4a16_dequant.restype = I
        L.w4a16_workspace_size.argtypes = [P, I, I, I]
        L.w4a16_workspace_size.restype = S
        L.w4a16_gemm.argtypes = [P, P, I, P, I, P, S, I, P]
        L.w4a16_gemm.restype = I
        L.w4a16_gemm_static.argtypes = [P, P, I, P, I, I, P]
        L.w4a16_gemm_static.restype = I
        PP = ctypes.POINTER(P)
        L.w4a16_comm_create.argtypes = [I, I, I, PP]
        L.w4a16_comm_destroy.argtypes = [P]
        L.w4a16_comm_flags.argtypes = [P, PP]
        L.w4a16_comm_set_peer_flags.argtypes = [P, I, P]
        L.w4a16_ipc_export.argtypes = [P, P]
        L.w4a16_ipc_open.argtypes = [P, I, PP]
        L.w4a16_ipc_close.argtypes = [P]
        L.w4a16_gemm_gather.argtypes = [P, P, P, I, P, I, I, I, P, S, P]
        for f in ("w4a16_comm_create", "w4a16_comm_destroy", "w4a16_comm_flags", "w4a16_comm_set_peer_flags",
                  "w4a16_ipc_export", "w4a16_ipc_open", "w4a16_ipc_close", "w4a16_gemm_gather"):
            getattr(L, f).restype = I
        L.w4a16_plan.argtypes = [P, I, I, I, IP]
        L.w4a16_plan.restype = I
        L.w4a16_plan_shape.argtypes = [I, I, I, I, I, I, I, I, IP, ctypes.POINTER(S)]
        L.w4a16_plan_shape.restype = I
        L.w4a16_info.argtypes = [P, IP]
        L.w4a16_info.restype = I
        L.w4a16_device_error.argtypes = [P, P, IP]
        L.w4a16_device_error.restype = I
        L.w4a16_last_error.argtypes = []
        L.w4a16_last_error.restype = ctypes.c_char_p
        L.w4a16_version.argtypes = []
        L.w4a16_version.restype = I
        _lib = L
        return L


_fast = None
_fast_tried = False


def torch_fast_path():
    """The C++ torch extension of the forward (``_w4a16_torch``, built in-tree by
    ``drofell_for_revision_b200.build``), or None where it was not built; both call the
    same C ABI and kernels."""
    global _fast, _fast_tried
    if not _fast_tried:
        _fast_tried = True
        lib()  # the extension links against the library: load it (and fail loudly) first
        try:
            from . import _w4a16_torch as mod
            _fast = mod
        except ImportError:
            _fast = None
    return _fast


def check(rc: int) -> None:
    if rc != W4A16_OK:
        msg = lib().w4a16_last_error()
        raise W4A16Error(rc, msg.decode() if msg else "")


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return DTYPE_FP16
    if dtype == torch.bfloat16:
        return DTYPE_BF16
    raise RuntimeError(f"x must be float16 or bfloat16, got {dtype}")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device | int | None = None) -> int:
    """cudaStream_t of the current torch stream on ``device`` (an int index is fastest)."""
    if _raw_stream is not None:
        if isinstance(device, torch.device):
            device = device.index if device.index is not None else torch.cuda.current_device()
        elif device is None:
            device = torch.cuda.current_device()
        return _raw_stream(device)
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (no CPU path exists)")


class Handle:
    """Owns one ``w4a16_matrix*``; destroyed with the Python object."""

    def __init__(self, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                 g_idx: torch.Tensor | None, device_index: int, repack: bool = True):
        for t, n in ((qweight, "qweight"), (qzeros, "qzeros"), (scales, "scales")):
            require_cuda(t, n)
            if not t.is_contiguous():
                raise RuntimeError(f"{n} must be contiguous")
        if qweight.dtype != torch.int32 or qzeros.dtype != torch.int32:
            raise RuntimeError("qweight and qzeros must be int32")
        if scales.dtype != torch.float16:
            raise RuntimeError("scales must be float16")
        K = qweight.shape[0] * 8
        N = qweight.shape[1]
        G = qzeros.shape[0]
        if qzeros.shape[1] * 8 != N or scales.shape[1] != N or scales.shape[0] != G:
            raise RuntimeError("qweight / qzeros / scales have incompatible shapes")
        self._g_idx_host = None
        gptr = None
        if g_idx is not None:
            gh = g_idx.detach().to("cpu", torch.int32).contiguous()
            if gh.numel() != K:
                raise RuntimeError("g_idx and qweight have incompatible shapes")
            self._g_idx_host = gh
            gptr = ctypes.c_void_p(gh.data_ptr())
        self.K, self.N, self.G = K, N, G
        self.device_index = device_index
        # keep the packed tensors alive: the handle holds raw pointers into them
        self._keep = (qweight, qzeros, scales)
        out = ctypes.c_void_p()
        # the environment switch W4A16_NO_REPACK=1 is honoured as by w4a16_create
        flags = 0 if repack and os.environ.get("W4A16_NO_REPACK", "0") in ("", "0") else CREATE_NO_REPACK
        with torch.cuda.device(device_index):
            check(lib().w4a16_create_ex(ctypes.c_void_p(qweight.data_ptr()), ctypes.c_void_p(qzeros.data_ptr()),
                                        ctypes.c_void_p(scales.data_ptr()), gptr, K, N, G, device_index, flags,
                                        ctypes.c_void_p(stream_ptr(device_index)), ctypes.byref(out)))
        self.ptr = out.value
        self._lib = lib()
        self._ws_need: dict = {}
        self._ws: torch.Tensor | None = None
        # Workspaces this handle has outgrown. They stay allocated for the handle's
        # lifetime: a CUDA graph captured while one of them was current still writes
        # into it on every replay, so returning it to the caching allocator would let
        # another tensor share that memory. Each replacement at least doubles the size,
        # so the retired ones together are smaller than the current one.
        self._ws_retired: list = []

    @property
    def as_int(self) -> int:
        return int(self.ptr)

    @property
    def symmetric(self) -> bool:
        """Every stored zero nibble is 7 (z = 8): the kernels skip the zero-point loads."""
        out = (ctypes.c_int * 4)()
        check(lib().w4a16_info(ctypes.c_void_p(self.ptr), out))
        return bool(out[3] & 2)

    def close(self) -> None:
        if getattr(self, "ptr", None):
            if _fast is not None:
                _fast.release(self.ptr)
            lib().w4a16_destroy(ctypes.c_void_p(self.ptr))
            self.ptr = None

    def __del__(self):  # pragma: no cover - interpreter shutdown ordering
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ ops
    def dequant(self, out: torch.Tensor) -> torch.Tensor:
        require_cuda(out, "out")
        if tuple(out.shape) != (self.K, self.N) or not out.is_contiguous():
            raise RuntimeError(f"out must be a contiguous [{self.K}, {self.N}] tensor")
        check(lib().w4a16_dequant(ctypes.c_void_p(self.ptr), ctypes.c_void_p(out.data_ptr()), dtype_code(out.dtype),
                                  ctypes.c_void_p(stream_ptr(out.device))))
        return out

    def workspace_size(self, M: int, dtype: torch.dtype, path: int = PATH_AUTO) -> int:
        return int(lib().w4a16_workspace_size(ctypes.c_void_p(self.ptr), M, dtype_code(dtype), path))

    def plan(self, M: int, dtype: torch.dtype = torch.float16, path: int = PATH_AUTO) -> tuple[int, int, int, int]:
        arr = (ctypes.c_int * 4)()
        check(lib().w4a16_plan(ctypes.c_void_p(self.ptr), M, dtype_code(dtype), path, arr))
        return tuple(arr)

    def _check_device(self, t: torch.Tensor, name: str) -> None:
        if t.device.index != self.device_index:
            raise RuntimeError(f"{name} is on {t.device}, the handle's weight on cuda:{self.device_index}")

    def _workspace(self, need: int, device: torch.device) -> torch.Tensor:
        """The handle's own workspace, grown (never shrunk or freed) to ``need`` bytes."""
        ws = self._ws
        if ws is None or ws.numel() < need:
            size = need if ws is None else max(need, 2 * ws.numel())
            if ws is not None:
                self._ws_retired.append(ws)
            ws = self._ws = torch.empty(size, dtype=torch.uint8, device=device)
        return ws

    def gemm(self, x: torch.Tensor, out: torch.Tensor, path: int = PATH_AUTO,
             workspace: torch.Tensor | None = None) -> torch.Tensor:
        """out[M, N] = x[M, K] @ W. x and out are contiguous CUDA tensors of the same dtype.

        Without ``workspace`` the handle keeps one, grown on demand and shared by all its
        calls, so calls on one Handle must not overlap on the GPU; pass a workspace per
        stream to overlap them."""
        if not (x.is_cuda and out.is_cuda):
            raise RuntimeError("x and out must be CUDA tensors (no CPU path exists)")
        if x.device.index != self.device_index or out.device.index != self.device_index:
            self._check_device(x, "x")
            self._check_device(out, "out")
        if x.dim() != 2 or x.shape[1] != self.K or not x.is_contiguous():
            raise RuntimeError("x and w have incompatible shapes (x must be contiguous [M, K])")
        M = x.shape[0]
        if out.shape[0] != M or out.shape[1] != self.N or out.dtype != x.dtype or not out.is_contiguous():
            raise RuntimeError("out must be a contiguous [M, N] tensor of x's dtype")
        dt = dtype_code(x.dtype)
        L = self._lib
        key = (M, dt, path)
        need = self._ws_need.get(key)
        if need is None:
            need = int(L.w4a16_workspace_size(self.ptr, M, dt, path))
            self._ws_need[key] = need
        ws_ptr, ws_bytes = None, 0
        if need > 0:
            if workspace is None:
                workspace = self._workspace(need, x.device)
            elif workspace.numel() * workspace.element_size() < need:
                raise RuntimeError(f"workspace of {workspace.numel() * workspace.element_size()} bytes < {need} "
                                   f"needed for M={M}")
            ws_ptr = workspace.data_ptr()
            ws_bytes = workspace.numel() * workspace.element_size()
        rc = L.w4a16_gemm(self.ptr, x.data_ptr(), M, out.data_ptr(), dt, ws_ptr, ws_bytes, path,
                          stream_ptr(self.device_index))
        if rc != W4A16_OK:
            check(rc)
        return out

    def gemm_static(self, x: torch.Tensor, out: torch.Tensor, path: int = PATH_AUTO) -> torch.Tensor:
        """``gemm`` with the library's fixed device scratch instead of a workspace
        (w4a16_gemm_static: allocates nothing; overlapping calls on a device race)."""
        require_cuda(x, "x")
        require_cuda(out, "out")
        self._check_device(x, "x")
        self._check_device(out, "out")
        if x.dim() != 2 or x.shape[1] != self.K or not x.is_contiguous():
            raise RuntimeError("x and w have incompatible shapes (x must be contiguous [M, K])")
        M = x.shape[0]
        if tuple(out.shape) != (M, self.N) or out.dtype != x.dtype or not out.is_contiguous():
            raise RuntimeError("out must be a contiguous [M, N] tensor of x's dtype")
        check(lib().w4a16_gemm_static(ctypes.c_void_p(self.ptr), ctypes.c_void_p(x.data_ptr()), M,
                                      ctypes.c_void_p(out.data_ptr()), dtype_code(x.dtype), path,
                                      ctypes.c_void_p(stream_ptr(self.device_index))))
        return out

    def gemm_gather(self, x: torch.Tensor, comm: "Comm", y_ptrs, ld: int, col0: int,
                    workspace: torch.Tensor | None = None) -> None:
        """This rank's columns of x @ W into every rank's full Y (w4a16_gemm_gather)."""
        if not x.is_cuda or x.dim() != 2 or x.shape[1] != self.K or not x.is_contiguous():
            raise RuntimeError("x must be a contiguous CUDA [M, K] tensor")
        self._check_device(x, "x")
        M = x.shape[0]
        dt = dtype_code(x.dtype)
        need = int(self._lib.w4a16_workspace_size(self.ptr, M, dt, PATH_AUTO))
        ws_ptr, ws_bytes = None, 0
        if need > 0:
            if workspace is None:
                workspace = self._workspace(need, x.device)
            ws_ptr = workspace.data_ptr()
            ws_bytes = workspace.numel() * workspace.element_size()
        arr = (ctypes.c_void_p * len(y_ptrs))(*y_ptrs)
        check(self._lib.w4a16_gemm_gather(self.ptr, comm.ptr, x.data_ptr(), M, arr, ld, col0, dt, ws_ptr, ws_bytes,
                                          stream_ptr(self.device_index)))

    def gemm_t(self, dy: torch.Tensor, out: torch.Tensor, workspace: torch.Tensor | None = None) -> torch.Tensor:
        """out[M, K] = dy[M, N] @ W^T (w4a16_gemm_t): the input gradient, in the caller's
        row order. Same workspace rules as ``gemm``."""
        if not (dy.is_cuda and out.is_cuda):
            raise RuntimeError("dy and out must be CUDA tensors (no CPU path exists)")
        self._check_device(dy, "dy")
        self._check_device(out, "out")
        if dy.dim() != 2 or dy.shape[1] != self.N or not dy.is_contiguous():
            raise RuntimeError("dy and w have incompatible shapes (dy must be contiguous [M, N])")
        M = dy.shape[0]
        if tuple(out.shape) != (M, self.K) or out.dtype != dy.dtype or not out.is_contiguous():
            raise RuntimeError("out must be a contiguous [M, K] tensor of dy's dtype")
        dt = dtype_code(dy.dtype)
        need = int(self._lib.w4a16_workspace_size_t(self.ptr, M, dt))
        ws_ptr, ws_bytes = None, 0
        if need > 0:
            if workspace is None:
                workspace = self._workspace(need, dy.device)
            elif workspace.numel() * workspace.element_size() < need:
                raise RuntimeError(f"workspace smaller than the {need} bytes needed for M={M}")
            ws_ptr = workspace.data_ptr()
            ws_bytes = workspace.numel() * workspace.element_size()
        check(self._lib.w4a16_gemm_t(self.ptr, dy.data_ptr(), M, out.data_ptr(), dt, ws_ptr, ws_bytes,
                                     stream_ptr(self.device_index)))
        return out

    def workspace_size_t(self, M: int, dtype: torch.dtype) -> int:
        return int(lib().w4a16_workspace_size_t(ctypes.c_void_p(self.ptr), M, dtype_code(dtype)))

    def device_error(self) -> int:
        v = ctypes.c_int(0)
        check(lib().w4a16_device_error(ctypes.c_void_p(self.ptr), ctypes.c_void_p(stream_ptr(self.device_index)),
                                       ctypes.byref(v)))
        return v.value


def _fp16_rows(t: torch.Tensor, name: str, cols: int | None = None) -> None:
    require_cuda(t, name)
    if t.dtype != torch.float16 or not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous float16 CUDA tensor")
    if cols is not None and t.shape[-1] != cols:
        raise RuntimeError(f"{name} has {t.shape[-1]} columns, {cols} expected")


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor) -> torch.Tensor:
    """out = RMSNorm(x; w, eps) row by row (w4a16_rms_norm), fp16."""
    K = x.shape[-1]
    for t, n in ((x, "x"), (w, "norm weight"), (out, "out")):
        _fp16_rows(t, n, K)
    check(lib().w4a16_rms_norm(x.data_ptr(), w.data_ptr(), float(eps), x.numel() // K, K, out.data_ptr(),
                               DTYPE_FP16, stream_ptr(x.device.index)))
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out = silu(gate) * up (w4a16_silu_mul), fp16; out may be gate."""
    N = gate.shape[-1]
    for t, n in ((gate, "gate"), (up, "up"), (out, "out")):
        _fp16_rows(t, n, N)
    check(lib().w4a16_silu_mul(gate.data_ptr(), up.data_ptr(), gate.numel() // N, N, out.data_ptr(), DTYPE_FP16,
                               stream_ptr(gate.device.index)))
    return out


def mlp_forward(gate: Handle, up: Handle, down: Handle, norm_w: torch.Tensor, eps: float, x: torch.Tensor,
                y: torch.Tensor, rms_out: torch.Tensor, gate_out: torch.Tensor, up_out: torch.Tensor) -> torch.Tensor:
    """y = down(silu(gate(r)) * up(r)), r = RMSNorm(x) into rms_out (w4a16_mlp_forward).
    gate_out / up_out are the block's scratch. The workspace, when one is needed, is the
    gate handle's own."""
    M = x.numel() // gate.K
    _fp16_rows(x, "x", gate.K)
    _fp16_rows(norm_w, "norm weight", gate.K)
    _fp16_rows(y, "y", down.N)
    _fp16_rows(rms_out, "rms_out", gate.K)
    _fp16_rows(gate_out, "gate_out", gate.N)
    _fp16_rows(up_out, "up_out", up.N)
    need = int(lib().w4a16_mlp_workspace_size(gate.ptr, up.ptr, down.ptr, M, DTYPE_FP16))
    ws = gate._workspace(need, x.device) if need > 0 else None
    check(lib().w4a16_mlp_forward(gate.ptr, up.ptr, down.ptr, norm_w.data_ptr(), float(eps), x.data_ptr(), M,
                                  y.data_ptr(), rms_out.data_ptr(), gate_out.data_ptr(), up_out.data_ptr(),
                                  DTYPE_FP16, ws.data_ptr() if ws is not None else None,
                                  ws.numel() if ws is not None else 0, stream_ptr(gate.device_index)))
    return y


def qkv_forward(q: Handle, k: Handle, v: Handle, norm_w: torch.Tensor, eps: float, x: torch.Tensor,
                rms_out: torch.Tensor, q_out: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor) -> None:
    """r = RMSNorm(x) into rms_out, then q_out, k_out, v_out = r Wq, r Wk, r Wv
    (w4a16_qkv_forward)."""
    M = x.numel() // q.K
    _fp16_rows(x, "x", q.K)
    _fp16_rows(norm_w, "norm weight", q.K)
    _fp16_rows(rms_out, "rms_out", q.K)
    _fp16_rows(q_out, "q_out", q.N)
    _fp16_rows(k_out, "k_out", k.N)
    _fp16_rows(v_out, "v_out", v.N)
    need = int(lib().w4a16_qkv_workspace_size(q.ptr, k.ptr, v.ptr, M, DTYPE_FP16))
    ws = q._workspace(need, x.device) if need > 0 else None
    check(lib().w4a16_qkv_forward(q.ptr, k.ptr, v.ptr, norm_w.data_ptr(), float(eps), x.data_ptr(), M,
                                  rms_out.data_ptr(), q_out.data_ptr(), k_out.data_ptr(), v_out.data_ptr(),
                                  DTYPE_FP16, ws.data_ptr() if ws is not None else None,
                                  ws.numel() if ws is not None else 0, stream_ptr(q.device_index)))


def plan_orientation(K: int, N: int, groups: int, M: int, dtype: torch.dtype = torch.float16,
                     path: int = PATH_AUTO, num_sms: int = 148, act_order: bool = False) -> str:
    """'natural' (128 tokens x 256 weight columns per MMA), 'swap' (128 weight columns x
    the token tile per MMA) or '' when the plan is a GEMV."""
    out = (ctypes.c_int * 5)()
    ws = ctypes.c_size_t(0)
    check(lib().w4a16_plan_shape(K, N, groups, 1 if act_order else 0, M, dtype_code(dtype), path, num_sms, out,
                                 ctypes.byref(ws)))
    if out[0] != KERN_EXACT:
        return ""
    return "natural" if out[4] & 2 else "swap"


def plan_shape(K: int, N: int, groups: int, M: int, dtype: torch.dtype = torch.float16, path: int = PATH_AUTO,
               num_sms: int = 148, act_order: bool = False) -> tuple[tuple[int, int, int, int], bool, int]:
    """The plan a handle of this shape would use on a GPU with ``num_sms`` SMs, without
    a GPU (w4a16_plan_shape): ((kernel, tile, splits, rows per pass or chunks per split),
    CUDA-core GEMV in its WIDE configuration, workspace bytes). ``plan_orientation``
    tells the tcgen05 GEMM's two orientations apart."""
    out = (ctypes.c_int * 5)()
    ws = ctypes.c_size_t(0)
    check(lib().w4a16_plan_shape(K, N, groups, 1 if act_order else 0, M, dtype_code(dtype), path, num_sms, out,
                                 ctypes.byref(ws)))
    return (out[0], out[1], out[2], out[3]), bool(out[4] & 1), ws.value


def ipc_export(t: torch.Tensor) -> bytes:
    """CUDA IPC handle (plus offset) of a CUDA tensor's memory, for another process."""
    require_cuda(t, "tensor")
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    check(lib().w4a16_ipc_export(ctypes.c_void_p(t.data_ptr()), buf))
    return buf.raw


def ipc_open(handle: bytes, device_index: int) -> int:
    """Map another process's export on this device; returns the device address."""
    out = ctypes.c_void_p()
    check(lib().w4a16_ipc_open(ctypes.c_char_p(handle), device_index, ctypes.byref(out)))
    return int(out.value)


def ipc_close(ptr: int) -> None:
    check(lib().w4a16_ipc_close(ctypes.c_void_p(ptr)))


class Comm:
    """One rank's flags and counters of a peer-memory gather group (w4a16_comm)."""

    def __init__(self, rank: int, world: int, device_index: int):
        out = ctypes.c_void_p()
        check(lib().w4a16_comm_create(rank, world, device_index, ctypes.byref(out)))
        self.ptr = out.value
        self.rank, self.world, self.device_index = rank, world, device_index
        self._opened: list = []

    def flags_handle(self) -> bytes:
        p = ctypes.c_void_p()
        check(lib().w4a16_comm_flags(ctypes.c_void_p(self.ptr), ctypes.byref(p)))
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(lib().w4a16_ipc_export(p, buf))
        return buf.raw

    def set_peer_flags(self, peer: int, handle: bytes) -> None:
        ptr = ipc_open(handle, self.device_index)
        self._opened.append(ptr)
        check(lib().w4a16_comm_set_peer_flags(ctypes.c_void_p(self.ptr), peer, ctypes.c_void_p(ptr)))

    def open(self, handle: bytes) -> int:
        ptr = ipc_open(handle, self.device_index)
        self._opened.append(ptr)
        return ptr

    def close(self) -> None:
        if getattr(self, "ptr", None):
            for p in self._opened:
                try:
                    ipc_close(p)
                except W4A16Error:
                    pass
            self._opened = []
            lib().w4a16_comm_destroy(ctypes.c_void_p(self.ptr))
            self.ptr = None

    def __del__(self):  # pragma: no cover - interpreter shutdown ordering
        try:
            self.close()
        except Exception:
            pass
