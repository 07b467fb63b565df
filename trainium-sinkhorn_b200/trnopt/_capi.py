"""ctypes binding of libtrnopt_cuda.so (the C ABI declared in include/trnopt_cuda.h).

There is no fallback: if the library is missing, importing this module raises ImportError telling how to build it,
and every wrapper raises TrnoptError when the C call returns a negative status. Tensors are passed as raw device
pointers with the current torch CUDA stream, so calls queue asynchronously like any other kernel on that stream.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("TRNOPT_CUDA_LIB", Path(__file__).resolve().parent / "libtrnopt_cuda.so"))

PATH_FFMA, PATH_TC = 0, 1


class TrnoptError(RuntimeError):
    """A negative status from the C ABI (argument, alignment, workspace, CUDA or device-flag error)."""


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built: run `python trainium-sinkhorn_b200/trnopt/_build.py` "
                          "(or __graft_entry__.build()); this package has no CPU fallback")
    return ctypes.CDLL(str(LIB_PATH))


lib = _load()

_P, _I, _F, _D, _Z = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_size_t
_SIGS = {
    "trnopt_version": (_I, []),
    "trnopt_status_string": (ctypes.c_char_p, [_I]),
    "trnopt_last_cuda_error": (_I, []),
    "trnopt_device_error_flags": (_I, [_P, ctypes.POINTER(_I)]),
    "trnopt_workspace_size": (_Z, [_I, _I, _I, _I]),
    "trnopt_workspace_init": (_I, [_P, _Z, _P]),
    "trnopt_half_step": (_I, [_P, _I, _P, _P, _P, _I, _P, _P, _I, _I, _I, _F, _F, _P, _P, _Z, _P]),
    "trnopt_row_lse": (_I, [_P, _I, _P, _I, _I, _I, _I, _P, _P, _Z, _P]),
    "trnopt_balanced_error": (_I, [_P, _P, _P, _I, _F, _P, _P]),
    "trnopt_max_change": (_I, [_P, _P, _I, _F, _P, _P]),
    "trnopt_pack_bytes": (_Z, [_I, _I]),
    "trnopt_pack_cloud": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "trnopt_half_step_tc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _F, _P, _P, _Z, _P]),
    "trnopt_static_scratch_bytes": (_Z, []),
    "trnopt_half_step_tc_static": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _F, _P, _P]),
    "trnopt_test_ex2_poly": (_I, [_P, _P, _I, _P]),
    "trnopt_sinkhorn_run": (_I, [_I, _P, _I, _P, _P, _P, _I, _I, _P, _I, _P, _P, _P, _I, _I, _I, _P, _P, _P, _I, _I,
                                 _F, _F, _F, _P, _Z, _P]),
    "trnopt_median_workspace_size": (_Z, []),
    "trnopt_median_cost": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _P, _Z, _P]),
    "trnopt_comm_handle_bytes": (_Z, []),
    "trnopt_comm_create": (_I, [_I, _I, _Z, ctypes.POINTER(_P), _P]),
    "trnopt_comm_open": (_I, [_P, _P]),
    "trnopt_comm_buffer": (_P, [_P]),
    "trnopt_comm_buffer_bytes": (_Z, [_P]),
    "trnopt_comm_epoch": (ctypes.c_ulonglong, [_P]),
    "trnopt_comm_arrive": (_I, [_P, _P]),
    "trnopt_comm_wait": (_I, [_P, _P]),
    "trnopt_comm_destroy": (_I, [_P]),
    "trnopt_sinkhorn_run_sharded": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _I, _I,
                                         _F, _F, _F, _P, _Z, _P]),
    "trnopt_cloud_stats_scratch_bytes": (_Z, [_I]),
    "trnopt_cloud_stats": (_I, [_P, _I, _P, _I, _I, _P, _P, _Z, _P]),
    "trnopt_prepare_cloud": (_I, [_P, _I, _I, _I, _P, _D, _P, _I, _P, _D, _P, _P, _P, _P, _P, _P, _P]),
    "trnopt_unshift": (_I, [_P, _P, _I, _P, _I, _P, _P]),
    "trnopt_recenter": (_I, [_P, _I, _I, _P, _P, _P]),
    "trnopt_solve_init": (_I, [_P, _P, _I, _D, _D, _D, _I, _I, _I, _I, _I, _F, _F, _I, _I, _I, _P]),
    "trnopt_sinkhorn_run_checked": (_I, [_I, _P, _I, _P, _P, _P, _I, _I, _P, _I, _P, _P, _P, _I, _I, _I, _P, _P, _P,
                                         _I, _I, _P, _P, _P, _Z, _P]),
    "trnopt_take_error_flags": (_I, [_P, _P]),
    "trnopt_plan_rows": (_I, [_P, _I, _P, _I, _I, _P, _P, _P, _P, _D, _P, _I, _P, _P]),
    "trnopt_plan_workspace_size": (_Z, [_I, _I]),
    "trnopt_plan_log_row_sums": (_I, [_P, _I, _P, _I, _I, _P, _P, _P, _P, _D, _P, _P, _Z, _P]),
}
for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype, _fn.argtypes = _res, _args


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib.trnopt_status_string(status).decode()
        extra = f" (cudaError {lib.trnopt_last_cuda_error()})" if status == -5 else ""
        raise TrnoptError(f"{what}: {msg}{extra}")


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t: torch.Tensor, name: str, dtype=torch.float32) -> None:
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous {dtype} CUDA tensor")


def workspace_size(rows: int, m: int, d: int, path: int = PATH_FFMA) -> int:
    return int(lib.trnopt_workspace_size(rows, m, d, path))


def new_workspace(nbytes: int, device) -> torch.Tensor:
    """A zeroed workspace from the torch caching allocator (256-byte aligned)."""
    ws = torch.empty(max(256, nbytes), dtype=torch.uint8, device=device)
    check(lib.trnopt_workspace_init(_ptr(ws), ws.numel(), _stream()), "trnopt_workspace_init")
    return ws


def half_step(xT, ldx, xsq, off, yT, ldy, gh, log_b, rows, m, d, eps, kappa, fh, ws) -> None:
    """Queue the FFMA fused half-step: fh[:rows] from the transposed clouds xT (d, ldx) and yT (d, ldy)."""
    check(lib.trnopt_half_step(_ptr(xT), ldx, _ptr(xsq), _ptr(off), _ptr(yT), ldy, _ptr(gh), _ptr(log_b), rows, m,
                               d, float(eps), float(kappa), _ptr(fh), _ptr(ws), ws.numel(), _stream()),
          "trnopt_half_step")


def pack_bytes(n: int, d: int) -> int:
    return int(lib.trnopt_pack_bytes(n, d))


def tc_supported(d: int) -> bool:
    return pack_bytes(1, d) > 0


def pack_cloud(xT: torch.Tensor, ld: int, n: int, d: int, scale_exp: int) -> torch.Tensor:
    """Split a transposed cloud (d, ld) into the FP16 [hi | lo] rows of the tensor-core path."""
    nbytes = pack_bytes(n, d)
    if nbytes == 0:
        raise ValueError(f"the tensor-core path does not support d = {d}")
    out = torch.empty(nbytes // 2, dtype=torch.float16, device=xT.device)
    check(lib.trnopt_pack_cloud(_ptr(xT), ld, n, d, int(scale_exp), _ptr(out), _stream()), "trnopt_pack_cloud")
    return out


def half_step_tc(xpack, xsq, off, ypack, gh, log_b, rows, m, d, sx, sy, eps, kappa, fh, ws) -> None:
    """Queue the tensor-core fused half-step on packed clouds."""
    check(lib.trnopt_half_step_tc(_ptr(xpack), _ptr(xsq), _ptr(off), _ptr(ypack), _ptr(gh), _ptr(log_b), rows, m, d,
                                  int(sx), int(sy), float(eps), float(kappa), _ptr(fh), _ptr(ws), ws.numel(),
                                  _stream()), "trnopt_half_step_tc")


def half_step_tc_static(xpack, xsq, off, ypack, gh, log_b, rows, m, d, sx, sy, eps, kappa, fh) -> None:
    """The tensor-core half-step with the library's static scratch instead of a workspace (allocates nothing)."""
    check(lib.trnopt_half_step_tc_static(_ptr(xpack), _ptr(xsq), _ptr(off), _ptr(ypack), _ptr(gh), _ptr(log_b), rows,
                                         m, d, int(sx), int(sy), float(eps), float(kappa), _ptr(fh), _stream()),
          "trnopt_half_step_tc_static")


def row_lse(xaT: torch.Tensor, yaT: torch.Tensor, ws: torch.Tensor | None = None) -> torch.Tensor:
    """lse_i = log sum_j exp(xa_i . ya_j) for xa_T (k, rows), ya_T (k, m) (the reference's row-LSE kernel)."""
    _need(xaT, "xa_T")
    _need(yaT, "ya_T")
    k, rows = xaT.shape
    m = yaT.shape[1]
    if yaT.shape[0] != k:
        raise ValueError("xa_T and ya_T need the same number of rows (contraction length)")
    xaT, ldx = _pad_ld(xaT)
    yaT, ldy = _pad_ld(yaT)
    if ws is None:
        ws = new_workspace(workspace_size(rows, m, k, PATH_FFMA), xaT.device)
    out = torch.empty(rows, dtype=torch.float32, device=xaT.device)
    check(lib.trnopt_row_lse(_ptr(xaT), ldx, _ptr(yaT), ldy, rows, m, k, _ptr(out), _ptr(ws), ws.numel(),
                             _stream()), "trnopt_row_lse")
    return out


def _pad_ld(t: torch.Tensor):
    """Copy a (k, n) matrix into one whose leading dimension is a multiple of 4 (the 16-byte row rule)."""
    k, n = t.shape
    ld = -(-n // 4) * 4
    if ld == n and t.data_ptr() % 16 == 0:
        return t, ld
    out = torch.zeros((k, ld), dtype=t.dtype, device=t.device)
    out[:, :n] = t
    return out, ld


def balanced_error(gh_old, gh_new, w, n, inv_eps, out) -> None:
    check(lib.trnopt_balanced_error(_ptr(gh_old), _ptr(gh_new), _ptr(w), n, float(inv_eps), _ptr(out), _stream()),
          "trnopt_balanced_error")


def max_change(gh_old, gh_new, n, inv_eps, out) -> None:
    check(lib.trnopt_max_change(_ptr(gh_old), _ptr(gh_new), n, float(inv_eps), _ptr(out), _stream()),
          "trnopt_max_change")


def median_cost(xc: torch.Tensor, yc: torch.Tensor, sqx: torch.Tensor, sqy: torch.Tensor) -> torch.Tensor:
    """Exact median of all clamped costs (float64 device scalar in a 1-element tensor)."""
    for t, nm in ((xc, "xc"), (yc, "yc"), (sqx, "sqx"), (sqy, "sqy")):
        _need(t, nm, torch.float64)
    n, d = xc.shape
    m = yc.shape[0]
    ws = torch.empty(int(lib.trnopt_median_workspace_size()), dtype=torch.uint8, device=xc.device)
    out = torch.empty(1, dtype=torch.float64, device=xc.device)
    check(lib.trnopt_median_cost(_ptr(xc), _ptr(yc), _ptr(sqx), _ptr(sqy), n, m, d, _ptr(out), _ptr(ws), ws.numel(),
                                 _stream()), "trnopt_median_cost")
    return out


def test_ex2_poly(x: torch.Tensor) -> torch.Tensor:
    """2^x through the library's FMA-pipe exp2 (self-test hook)."""
    _need(x, "x")
    out = torch.empty_like(x)
    check(lib.trnopt_test_ex2_poly(_ptr(x), _ptr(out), x.numel(), _stream()), "trnopt_test_ex2_poly")
    return out


def sinkhorn_run(path, x_op, ldx, xsq, xoff, log_a, nx, sx, y_op, ldy, ysq, yoff, log_b, ny, sy, d, g0, g1, fh,
                 start_parity, n_iter, eps, kappa_x, kappa_y, ws) -> None:
    """Queue n_iter iterations (f then g half-step each) with ping-pong g buffers g0 / g1 in one C call."""
    check(lib.trnopt_sinkhorn_run(path, _ptr(x_op), ldx, _ptr(xsq), _ptr(xoff), _ptr(log_a), nx, int(sx), _ptr(y_op),
                                  ldy, _ptr(ysq), _ptr(yoff), _ptr(log_b), ny, int(sy), d, _ptr(g0), _ptr(g1),
                                  _ptr(fh), int(start_parity), int(n_iter), float(eps), float(kappa_x),
                                  float(kappa_y), _ptr(ws), ws.numel(), _stream()), "trnopt_sinkhorn_run")


def _plan_args(x, y, f, g, log_a, log_b):
    _need(x, "x", torch.float64)
    _need(y, "y", torch.float64)
    if x.dim() != 2 or y.dim() != 2 or x.shape[1] != y.shape[1]:
        raise ValueError("x (n, d) and y (m, d) must share d")
    for t, nm, n in ((f, "f", x.shape[0]), (g, "g", y.shape[0]), (log_a, "log_a", x.shape[0]),
                     (log_b, "log_b", y.shape[0])):
        if t is not None:
            _need(t, nm, torch.float64)
            if t.shape != (n,):
                raise ValueError(f"{nm} must have shape ({n},)")


def plan_rows(x, y, f, g, log_a, log_b, eps, rows: torch.Tensor) -> torch.Tensor:
    """Rows P[rows, :] of P = exp(log_a + log_b^T + (f + g^T - C) / eps), float64 (n, d) / (m, d) clouds."""
    _plan_args(x, y, f, g, log_a, log_b)
    _need(rows, "rows", torch.int32)
    n, d = x.shape
    m = y.shape[0]
    out = torch.empty((rows.numel(), m), dtype=torch.float64, device=x.device)
    check(lib.trnopt_plan_rows(_ptr(x), n, _ptr(y), m, d, _ptr(f), _ptr(g), _ptr(log_a), _ptr(log_b), float(eps),
                               _ptr(rows), rows.numel(), _ptr(out), _stream()), "trnopt_plan_rows")
    return out


def plan_log_row_sums(x, y, f, g, log_a, log_b, eps) -> torch.Tensor:
    """log sum_j P_ij for every row i, float64."""
    _plan_args(x, y, f, g, log_a, log_b)
    n, d = x.shape
    m = y.shape[0]
    ws = torch.empty(max(8, int(lib.trnopt_plan_workspace_size(n, m))), dtype=torch.uint8, device=x.device)
    out = torch.empty(n, dtype=torch.float64, device=x.device)
    check(lib.trnopt_plan_log_row_sums(_ptr(x), n, _ptr(y), m, d, _ptr(f), _ptr(g), _ptr(log_a), _ptr(log_b),
                                       float(eps), _ptr(out), _ptr(ws), ws.numel(), _stream()),
          "trnopt_plan_log_row_sums")
    return out


def sinkhorn_run_sharded(comm, xpack, xsq, xoff, log_a, nx, sx, ypack, ysq, yoff, log_b, ny, sy, d, g0, g1, fh,
                         start_parity, n_iter, eps, kappa_x, kappa_y, ws) -> None:
    """Queue n_iter iterations over row shards, each half-step publishing its rows to every rank (comm: a
    trnopt_comm handle; g0, g1, fh in its buffer)."""
    check(lib.trnopt_sinkhorn_run_sharded(comm, _ptr(xpack), _ptr(xsq), _ptr(xoff), _ptr(log_a), nx, int(sx),
                                          _ptr(ypack), _ptr(ysq), _ptr(yoff), _ptr(log_b), ny, int(sy), d, _ptr(g0),
                                          _ptr(g1), _ptr(fh), int(start_parity), int(n_iter), float(eps),
                                          float(kappa_x), float(kappa_y), _ptr(ws), ws.numel(), _stream()),
          "trnopt_sinkhorn_run_sharded")


def device_error_flags() -> int:
    flags = ctypes.c_int(0)
    check(lib.trnopt_device_error_flags(_stream(), ctypes.byref(flags)), "trnopt_device_error_flags")
    return int(flags.value)


def cloud_stats_scratch(d: int, device) -> torch.Tensor:
    """Scratch of trnopt_cloud_stats, zeroed once (the kernel leaves it zeroed)."""
    nbytes = int(lib.trnopt_cloud_stats_scratch_bytes(d))
    if nbytes == 0:
        raise ValueError(f"cloud statistics support 1 <= d <= 128, not {d}")
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def cloud_stats(x: torch.Tensor, y: torch.Tensor, stats: torch.Tensor, scratch: torch.Tensor) -> None:
    """stats (2, 3, d) float64 <- per-coordinate (sum, min, max) of the float64 clouds x (n, d) and y (m, d)."""
    n, d = x.shape
    check(lib.trnopt_cloud_stats(_ptr(x), n, _ptr(y), y.shape[0], d, _ptr(stats), _ptr(scratch), scratch.numel(),
                                 _stream()), "trnopt_cloud_stats")


def prepare_cloud(pts: torch.Tensor, n: int, npad: int, center, r: float, shift, scale_exp: int, log_w, lw_uniform,
                  off, packed, xT, vec, sq64, gh0) -> None:
    """One cloud in the half-step layout (trnopt_prepare_cloud); center / shift are host float64 arrays."""
    import numpy as np
    d = pts.shape[1]
    c = np.ascontiguousarray(center, dtype=np.float64)
    sh = np.ascontiguousarray(shift, dtype=np.float64)
    check(lib.trnopt_prepare_cloud(_ptr(pts), n, d, npad, c.ctypes.data_as(_P), float(r), sh.ctypes.data_as(_P),
                                   int(scale_exp), _ptr(log_w), float(lw_uniform), _ptr(off), _ptr(packed),
                                   _ptr(xT), _ptr(vec), _ptr(sq64), _ptr(gh0), _stream()), "trnopt_prepare_cloud")


def unshift(h, sq, n: int, out, gauge=None, sign: int = 1) -> None:
    """out[:n] = h[:n] + sq[:n] + sign * gauge[0] in float64 (device tensors; out may be a view into a larger
    buffer; gauge None = 0)."""
    check(lib.trnopt_unshift(_ptr(h), _ptr(sq), n, _ptr(gauge), int(sign), _ptr(out), _stream()), "trnopt_unshift")


def recenter(gh, n: int, npad: int, gauge, state=None) -> None:
    """Balanced solves: gh -= K (its float32-rounded mean over the first n entries), gauge[0] += K; nothing once a
    solve state (if given) is done."""
    check(lib.trnopt_recenter(_ptr(gh), n, npad, _ptr(gauge), _ptr(state), _stream()), "trnopt_recenter")


MAX_STAGES = 32


class SolveState(ctypes.Structure):
    """Host mirror of TrnoptSolveState (include/trnopt_cuda.h), to read a copy of the device state."""
    _fields_ = [("stage_eps", _D * (MAX_STAGES + 1)), ("rho", _D * 2), ("tol", _F), ("stage_tol", _F),
                ("n_stages", _I), ("check_every", _I), ("max_iters", _I), ("stage_max_iters", _I),
                ("fixed_iters", _I), ("balanced", _I), ("sched_len", _I), ("n_real", _I), ("npad", _I),
                ("eps", _F), ("kappa", _F * 2), ("dot2", _F), ("gh2", _F),
                ("it", _I), ("stage", _I), ("stage_it", _I), ("done", _I), ("converged", _I), ("err", _F),
                ("stage_iters", _I * (MAX_STAGES + 1))]


def solve_init(state, stages, final_eps, rho_x, rho_y, check_every, max_iters, stage_max_iters, fixed_iters,
               sched_len, tol, stage_tol, n_real, npad, it0) -> None:
    """Write the plan and starting counters into a device TrnoptSolveState (state: a CUDA uint8 tensor)."""
    import numpy as np
    st = np.ascontiguousarray(stages if len(stages) else [0.0], dtype=np.float64)
    check(lib.trnopt_solve_init(_ptr(state), st.ctypes.data_as(_P), len(stages), float(final_eps),
                                float(-1.0 if rho_x is None else rho_x), float(-1.0 if rho_y is None else rho_y),
                                int(check_every), int(max_iters), int(stage_max_iters), int(bool(fixed_iters)),
                                int(sched_len), float(tol), float(stage_tol), int(n_real), int(npad), int(it0),
                                _stream()), "trnopt_solve_init")


def sinkhorn_run_checked(path, x_op, ldx, xsq, xoff, log_a, nx, sx, y_op, ldy, ysq, yoff, log_b, ny, sy, d, g0, g1,
                         fh, start_parity, n_iter, state, w_y, ws) -> None:
    """Queue n_iter iterations at the solve state's current eps stage, then the check at their end."""
    check(lib.trnopt_sinkhorn_run_checked(path, _ptr(x_op), ldx, _ptr(xsq), _ptr(xoff), _ptr(log_a), nx, int(sx),
                                          _ptr(y_op), ldy, _ptr(ysq), _ptr(yoff), _ptr(log_b), ny, int(sy), d,
                                          _ptr(g0), _ptr(g1), _ptr(fh), int(start_parity), int(n_iter), _ptr(state),
                                          _ptr(w_y), _ptr(ws), ws.numel(), _stream()), "trnopt_sinkhorn_run_checked")


def take_error_flags(out) -> None:
    """out[0] <- the device error word (cleared), asynchronously."""
    check(lib.trnopt_take_error_flags(_ptr(out), _stream()), "trnopt_take_error_flags")
