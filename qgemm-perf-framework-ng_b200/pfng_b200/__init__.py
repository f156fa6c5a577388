"""Python binding of libpfng_b200 (the C ABI in include/pfng_b200.h).

The library computes perf-framework-ng's hot path on a B200:
``C[m][n] = A[m][k] . W[n][k]^T`` for q4_0 x q8_0, q4_K x q8_K and
iq2_xxs x q8_K, plus the fp32 -> q8_0 / q8_K / q4_0 / q4_K quantizers.  This
module is plumbing: torch tensors hold device memory and streams, every
computation is a call into the shared library.  There is no CPU path; if the
library is not built, importing the functions raises immediately.

Block arrays are passed as flat ``torch.uint8`` tensors in the ggml wire
layout (bench/llama_reference and include/ggml.h of the reference); the
``*_BYTES`` constants give the size of one block.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import re

PACKAGE_DIR = pathlib.Path(__file__).resolve().parent.parent
REPO_ROOT = PACKAGE_DIR.parent
LIB_PATH = PACKAGE_DIR / "libpfng_b200.so"
HEADER_PATH = REPO_ROOT / "include" / "pfng_b200.h"

Q4_0, Q4_K, IQ2_XXS, Q4_0_PLANAR = 0, 1, 2, 3
WTYPES = {"q4_0": Q4_0, "q4_K": Q4_K, "iq2_xxs": IQ2_XXS, "q4_0_planar": Q4_0_PLANAR}
PATH_AUTO, PATH_GEMV, PATH_MMA, PATH_SIMPLE = 0, 1, 2, 3
PATHS = {"auto": PATH_AUTO, "gemv": PATH_GEMV, "mma": PATH_MMA, "simple": PATH_SIMPLE}

Q4_0_BYTES, Q8_0_BYTES, Q4_K_BYTES, Q8_K_BYTES, IQ2_XXS_BYTES = 18, 34, 144, 292, 66
# weight type -> (weight block bytes, weight block k, activation block bytes, activation block k)
LAYOUT = {
    Q4_0: (Q4_0_BYTES, 32, Q8_0_BYTES, 32),
    Q4_K: (Q4_K_BYTES, 256, Q8_K_BYTES, 256),
    IQ2_XXS: (IQ2_XXS_BYTES, 256, Q8_K_BYTES, 256),
    Q4_0_PLANAR: (Q4_0_BYTES, 32, Q8_0_BYTES, 32),  # same bytes per row as q4_0, reordered
}

OUT_F32, OUT_F16, OUT_BF16, OUT_Q8_0 = 0, 1, 2, 3
OUT_FORMATS = {"f32": OUT_F32, "f16": OUT_F16, "bf16": OUT_BF16, "q8_0": OUT_Q8_0}

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_KERNEL_TIMEOUT = -6
OVERLAP_WEIGHTS = 1


class PfngError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded shared library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `make -C {PACKAGE_DIR}` "
                "(or __graft_entry__.build()); there is no fallback implementation")
        _lib = ctypes.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    P, I64, I, S = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
    L.pfng_b200_version.restype = I
    L.pfng_b200_status_string.restype = ctypes.c_char_p
    L.pfng_b200_status_string.argtypes = [I]
    L.pfng_b200_check_kernel_error.restype = I
    L.pfng_b200_check_kernel_error.argtypes = [P]
    for q in ("q8_0", "q8_K", "q4_0", "q4_K"):
        f = getattr(L, f"pfng_b200_quantize_{q}")
        f.restype = I
        f.argtypes = [P, I64, P, I64, I64, P]
    for name in ("mm_workspace_size", "compute_workspace_size"):
        f = getattr(L, f"pfng_b200_{name}")
        f.restype = S
        f.argtypes = [I, I64, I64, I64, I]
    for t in ("q4_0_q8_0", "q4_K_q8_K", "iq2_xxs_q8_K", "q4_0p_q8_0"):
        f = getattr(L, f"pfng_b200_mm_{t}")
        f.restype = I
        f.argtypes = [P, P, P, I64, I64, I64, I64, P, S, I, P]
        f = getattr(L, f"pfng_b200_partials_{t}")
        f.restype = I
        f.argtypes = [P, P, P, I64, I64, I64, P, S, I, P]
    for t in ("q4_0", "q4_K", "iq2_xxs", "q4_0p"):
        f = getattr(L, f"pfng_b200_compute_{t}")
        f.restype = I
        f.argtypes = [P, P, I64, P, I64, I64, I64, I64, P, S, I, P]
    for name in ("mm_out_workspace_size", "compute_out_workspace_size"):
        f = getattr(L, f"pfng_b200_{name}")
        f.restype = S
        f.argtypes = [I, I, I64, I64, I64, I]
    L.pfng_b200_mm_out.restype = I
    L.pfng_b200_mm_out.argtypes = [I, P, P, P, I, I64, I64, I64, I64, P, S, I, P]
    L.pfng_b200_compute_out.restype = I
    L.pfng_b200_compute_out.argtypes = [I, P, P, I64, P, I, I64, I64, I64, I64, P, S, I, P]
    for name in ("pack_q4_0_planar", "unpack_q4_0_planar"):
        f = getattr(L, f"pfng_b200_{name}")
        f.restype = I
        f.argtypes = [P, P, I64, I64, P]
    L.pfng_b200_compute_grouped.restype = I
    L.pfng_b200_compute_grouped.argtypes = [I, I, ctypes.POINTER(P), ctypes.POINTER(I64), ctypes.POINTER(P),
                                            ctypes.POINTER(I64), P, I64, I64, I64, ctypes.c_uint, P]
    L.pfng_b200_shard_rows.restype = I
    L.pfng_b200_shard_rows.argtypes = [I64, I, I, I64, ctypes.POINTER(I64), ctypes.POINTER(I64)]
    L.pfng_b200_unshard_columns.restype = I
    L.pfng_b200_unshard_columns.argtypes = [P, P, I64, I64, I64, I, I64, I64, P]
    L.pfng_b200_compute_gather.restype = I
    L.pfng_b200_compute_gather.argtypes = [I, P, P, I64, ctypes.POINTER(P), I, I64, I64, I64, I64, P, S, I, P]
    L.pfng_b200_mm_gather.restype = I
    L.pfng_b200_mm_gather.argtypes = [I, P, P, ctypes.POINTER(P), I, I64, I64, I64, I64, P, S, I, P]
    L.pfng_b200_ipc_alloc.restype = I
    L.pfng_b200_ipc_alloc.argtypes = [S, ctypes.POINTER(P), P]
    L.pfng_b200_ipc_open.restype = I
    L.pfng_b200_ipc_open.argtypes = [P, ctypes.POINTER(P)]
    for name in ("ipc_free", "ipc_close"):
        f = getattr(L, f"pfng_b200_{name}")
        f.restype = I
        f.argtypes = [P]
    L.pfng_b200_prepared_bytes.restype = S
    L.pfng_b200_prepared_bytes.argtypes = [I, I64, I64]
    L.pfng_b200_prepare_activations.restype = I
    L.pfng_b200_prepare_activations.argtypes = [I, P, I64, P, S, I64, I64, P]
    L.pfng_b200_mm_prepared_workspace_size.restype = S
    L.pfng_b200_mm_prepared_workspace_size.argtypes = [I, I64, I64, I64]
    L.pfng_b200_mm_prepared.restype = I
    L.pfng_b200_mm_prepared.argtypes = [I, P, P, P, I64, I64, I64, I64, P, S, P]
    L.pfng_b200_selftest_wait.restype = I
    L.pfng_b200_selftest_wait.argtypes = [ctypes.c_uint, I, P, P]


def header_functions() -> list[str]:
    """Names of every function include/pfng_b200.h declares."""
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"\b(pfng_b200_[a-zA-Z0-9_]+)\s*\(", text)))


def status_string(status: int) -> str:
    return lib().pfng_b200_status_string(status).decode()


def _check(status: int, what: str) -> None:
    if status != OK:
        raise PfngError(status, what)


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _suffix(wtype: int) -> str:
    return {Q4_0: "q4_0_q8_0", Q4_K: "q4_K_q8_K", IQ2_XXS: "iq2_xxs_q8_K", Q4_0_PLANAR: "q4_0p_q8_0"}[wtype]


def _wt(wtype) -> int:
    return WTYPES[wtype] if isinstance(wtype, str) else int(wtype)


def _path(path) -> int:
    return PATHS[path] if isinstance(path, str) else int(path)


# ---------------------------------------------------------------- quantizers
def _quantize(kind: str, x, qk: int, block_bytes: int, out=None, stream=None):
    import torch
    rows, k = x.shape
    if out is None:
        out = torch.empty(rows * (k // qk) * block_bytes, dtype=torch.uint8, device=x.device)
    _check(getattr(lib(), f"pfng_b200_quantize_{kind}")(
        _ptr(x), x.stride(0), _ptr(out), rows, k, _stream(stream)), f"quantize_{kind}")
    return out


def quantize_q8_0(x, out=None, stream=None):
    """fp32 [m][k] -> block_q8_0 bytes (reference llama_reference.cpp:38-52)."""
    return _quantize("q8_0", x, 32, Q8_0_BYTES, out, stream)


def quantize_q8_K(x, out=None, stream=None):
    """fp32 [m][k] -> block_q8_K bytes (reference llama_reference.cpp:54-70)."""
    return _quantize("q8_K", x, 256, Q8_K_BYTES, out, stream)


def quantize_q4_0(x, out=None, stream=None):
    """fp32 [n][k] weights -> block_q4_0 bytes (reference llama_reference.cpp:13-36)."""
    return _quantize("q4_0", x, 32, Q4_0_BYTES, out, stream)


def quantize_q4_K(x, out=None, stream=None):
    """fp32 [n][k] weights -> block_q4_K bytes (reference llama_reference.cpp:72-111)."""
    return _quantize("q4_K", x, 256, Q4_K_BYTES, out, stream)


def quantize_activation(wtype, x, out=None, stream=None):
    q8_0 = _wt(wtype) in (Q4_0, Q4_0_PLANAR)
    return quantize_q8_0(x, out, stream) if q8_0 else quantize_q8_K(x, out, stream)


def pack_q4_0_planar(w, n: int, k: int, out=None, stream=None):
    """block_q4_0 bytes [n][k/32] -> the planar row layout (same size; k % 256 == 0)."""
    import torch
    if out is None:
        out = torch.empty(n * (k // 32) * Q4_0_BYTES, dtype=torch.uint8, device=w.device)
    _check(lib().pfng_b200_pack_q4_0_planar(_ptr(w), _ptr(out), n, k, _stream(stream)), "pack_q4_0_planar")
    return out


def unpack_q4_0_planar(wp, n: int, k: int, out=None, stream=None):
    """Planar row layout -> block_q4_0 bytes (the inverse of pack_q4_0_planar)."""
    import torch
    if out is None:
        out = torch.empty(n * (k // 32) * Q4_0_BYTES, dtype=torch.uint8, device=wp.device)
    _check(lib().pfng_b200_unpack_q4_0_planar(_ptr(wp), _ptr(out), n, k, _stream(stream)), "unpack_q4_0_planar")
    return out


# ------------------------------------------------------------------- matmul
def mm_workspace_size(wtype, m: int, n: int, k: int, path="auto") -> int:
    return lib().pfng_b200_mm_workspace_size(_wt(wtype), m, n, k, _path(path))


def compute_workspace_size(wtype, m: int, n: int, k: int, path="auto") -> int:
    return lib().pfng_b200_compute_workspace_size(_wt(wtype), m, n, k, _path(path))


def _workspace(nbytes: int, device, workspace):
    import torch
    if nbytes == 0:
        return workspace
    if workspace is not None and workspace.numel() >= nbytes:
        return workspace
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def mm(wtype, w, a, m: int, n: int, k: int, out=None, path="auto", workspace=None, stream=None):
    """C = A . W^T with pre-quantized activations `a` (q8_0 or q8_K bytes)."""
    import torch
    wt, p = _wt(wtype), _path(path)
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=w.device)
    ws = _workspace(mm_workspace_size(wt, m, n, k, p), w.device, workspace)
    nbytes = 0 if ws is None else ws.numel()
    _check(getattr(lib(), f"pfng_b200_mm_{_suffix(wt)}")(
        _ptr(w), _ptr(a), _ptr(out), m, n, k, out.stride(0), _ptr(ws), nbytes, p, _stream(stream)),
        f"mm_{_suffix(wt)}")
    return out


def compute(wtype, w, x, n: int, out=None, path="auto", workspace=None, stream=None):
    """The reference's compute(): quantize fp32 activations x [m][k], then C = A . W^T."""
    import torch
    wt, p = _wt(wtype), _path(path)
    m, k = x.shape
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=w.device)
    ws = _workspace(compute_workspace_size(wt, m, n, k, p), w.device, workspace)
    nbytes = 0 if ws is None else ws.numel()
    name = {Q4_0: "q4_0", Q4_K: "q4_K", IQ2_XXS: "iq2_xxs", Q4_0_PLANAR: "q4_0p"}[wt]
    _check(getattr(lib(), f"pfng_b200_compute_{name}")(
        _ptr(w), _ptr(x), x.stride(0), _ptr(out), m, n, k, out.stride(0), _ptr(ws), nbytes, p,
        _stream(stream)), f"compute_{name}")
    return out


def _fmt(out_format) -> int:
    return OUT_FORMATS[out_format] if isinstance(out_format, str) else int(out_format)


def _out_tensor(fmt: int, m: int, n: int, device):
    import torch
    if fmt == OUT_Q8_0:
        return torch.empty(m * (n // 32) * Q8_0_BYTES, dtype=torch.uint8, device=device)
    dt = {OUT_F32: torch.float32, OUT_F16: torch.float16, OUT_BF16: torch.bfloat16}[fmt]
    return torch.empty((m, n), dtype=dt, device=device)


def _ldo(fmt: int, out, n: int) -> int:
    return n // 32 if fmt == OUT_Q8_0 else out.stride(0)


def mm_out(wtype, w, a, m: int, n: int, k: int, out_format, out=None, path="auto", workspace=None, stream=None):
    """mm() with the result written as fp32 / fp16 / bf16 or q8_0 blocks along n (fused epilogue)."""
    wt, p, fmt = _wt(wtype), _path(path), _fmt(out_format)
    if out is None:
        out = _out_tensor(fmt, m, n, w.device)
    ws = _workspace(lib().pfng_b200_mm_out_workspace_size(wt, fmt, m, n, k, p), w.device, workspace)
    nbytes = 0 if ws is None else ws.numel()
    _check(lib().pfng_b200_mm_out(wt, _ptr(w), _ptr(a), _ptr(out), fmt, _ldo(fmt, out, n), m, n, k, _ptr(ws),
                                  nbytes, p, _stream(stream)), "mm_out")
    return out


def compute_out(wtype, w, x, n: int, out_format, out=None, path="auto", workspace=None, stream=None):
    """compute() with the result written as fp32 / fp16 / bf16 or q8_0 blocks along n (fused epilogue)."""
    wt, p, fmt = _wt(wtype), _path(path), _fmt(out_format)
    m, k = x.shape
    if out is None:
        out = _out_tensor(fmt, m, n, w.device)
    ws = _workspace(lib().pfng_b200_compute_out_workspace_size(wt, fmt, m, n, k, p), w.device, workspace)
    nbytes = 0 if ws is None else ws.numel()
    _check(lib().pfng_b200_compute_out(wt, _ptr(w), _ptr(x), x.stride(0), _ptr(out), fmt, _ldo(fmt, out, n), m, n,
                                       k, _ptr(ws), nbytes, p, _stream(stream)), "compute_out")
    return out


class GroupedCall:
    """Pre-marshalled arguments of pfng_b200_compute_grouped (several weight
    matrices sharing one activation), reusable across calls and graph capture."""

    def __init__(self, wtype, weights, ns, outs, x, overlap_weights=False):
        count = len(weights)
        self.flags = OVERLAP_WEIGHTS if overlap_weights else 0
        self.wtype = _wt(wtype)
        self.count = count
        self.w = (ctypes.c_void_p * count)(*[t.data_ptr() for t in weights])
        self.n = (ctypes.c_int64 * count)(*ns)
        self.c = (ctypes.c_void_p * count)(*[o.data_ptr() for o in outs])
        self.ldc = (ctypes.c_int64 * count)(*[o.stride(0) for o in outs])
        self.x = x
        self.keep = (weights, outs)

    def __call__(self, x=None, stream=None):
        x = self.x if x is None else x
        m, k = x.shape
        _check(lib().pfng_b200_compute_grouped(self.wtype, self.count, self.w, self.n, self.c, self.ldc,
                                               _ptr(x), x.stride(0), m, k, self.flags, _stream(stream)),
               "compute_grouped")


def compute_grouped(wtype, weights, x, ns, outs=None, overlap_weights=False, stream=None):
    """C_g = quantize(x) . W_g^T for several weight matrices in one launch."""
    import torch
    m = x.shape[0]
    if outs is None:
        outs = [torch.empty((m, n), dtype=torch.float32, device=x.device) for n in ns]
    GroupedCall(wtype, weights, ns, outs, x, overlap_weights)(stream=stream)
    return outs


def prepare_activations(wtype, x, out=None, stream=None):
    """fp32 x [m][k] (row stride x.stride(0)) quantized once into the
    tensor-core GEMM's operand layout (pfng_b200_prepare_activations); the
    result is a flat uint8 tensor for mm_prepared."""
    import torch
    wt = _wt(wtype)
    m, k = x.shape
    nbytes = lib().pfng_b200_prepared_bytes(wt, m, k)
    if nbytes == 0:
        raise PfngError(-2, "prepared_bytes")
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    _check(lib().pfng_b200_prepare_activations(wt, _ptr(x), x.stride(0), _ptr(out), out.numel(), m, k,
                                               _stream(stream)), "prepare_activations")
    return out


def mm_prepared_workspace_size(wtype, m: int, n: int, k: int) -> int:
    return lib().pfng_b200_mm_prepared_workspace_size(_wt(wtype), m, n, k)


def mm_prepared(wtype, w, prepared, m: int, n: int, k: int, out=None, workspace=None, stream=None):
    """C [m][n] = prepared activations . W^T: the tensor-core GEMM alone
    (pfng_b200_mm_prepared).  workspace=None allocates the split-k tiles
    the shape needs; pass a zero-size tensor to run unsplit."""
    import torch
    wt = _wt(wtype)
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=w.device)
    ws = _workspace(mm_prepared_workspace_size(wt, m, n, k), w.device, None) if workspace is None else workspace
    nbytes = 0 if ws is None else ws.numel()
    _check(lib().pfng_b200_mm_prepared(wt, _ptr(w), _ptr(prepared), _ptr(out), m, n, k, out.stride(0), _ptr(ws),
                                       nbytes, _stream(stream)), "mm_prepared")
    return out


def partials(wtype, w, a, m: int, n: int, k: int, path="auto", workspace=None, stream=None):
    """int32 [m][n][k/32] integer sub-block dot products of the chosen kernel path."""
    import torch
    wt, p = _wt(wtype), _path(path)
    out = torch.empty((m, n, k // 32), dtype=torch.int32, device=w.device)
    ws = _workspace(mm_workspace_size(wt, m, n, k, p), w.device, workspace)
    nbytes = 0 if ws is None else ws.numel()
    _check(getattr(lib(), f"pfng_b200_partials_{_suffix(wt)}")(
        _ptr(w), _ptr(a), _ptr(out), m, n, k, _ptr(ws), nbytes, p, _stream(stream)),
        f"partials_{_suffix(wt)}")
    return out


def check_kernel_error(stream=None) -> None:
    _check(lib().pfng_b200_check_kernel_error(_stream(stream)), "kernel error word")


def selftest_wait(attempts: int, skip_arrive: bool, stream=None):
    """Run the bounded-wait self-test kernel (pfng_b200_selftest_wait) and
    return (completed, status): whether the consumer's wait succeeded, and
    what pfng_b200_check_kernel_error reported afterwards (the error word is
    read and cleared)."""
    import torch
    done = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    _check(lib().pfng_b200_selftest_wait(attempts, 1 if skip_arrive else 0, _ptr(done), _stream(stream)),
           "selftest_wait")
    status = lib().pfng_b200_check_kernel_error(_stream(stream))
    return int(done.item()), status


# ----------------------------------------------------------------- sharding
def shard_rows(n: int, world: int, rank: int, granule: int) -> tuple[int, int]:
    b, e = ctypes.c_int64(0), ctypes.c_int64(0)
    _check(lib().pfng_b200_shard_rows(n, world, rank, granule, ctypes.byref(b), ctypes.byref(e)),
           "shard_rows")
    return b.value, e.value


def unshard_columns(slices, m: int, n: int, world: int, granule: int, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=slices.device)
    width = slices.shape[-1]
    _check(lib().pfng_b200_unshard_columns(_ptr(slices), _ptr(out), m, n, out.stride(0), world, granule,
                                           width, _stream(stream)), "unshard_columns")
    return out


# ------------------------------------------- fused all-gather of C over NVLink
MAX_DESTINATIONS = 8
IPC_HANDLE_BYTES = 64


def compute_gather(wtype, w, x, n: int, destinations, ldd: int, path="auto", workspace=None, stream=None) -> None:
    """compute() storing C [m][n] to every device pointer in `destinations` (row stride `ldd` floats):
    the first is typically this GPU's C, the others other GPUs' C opened with ipc_open.  The call
    does not wait for other ranks; order them (a barrier or collective on the stream) before C is read."""
    wt, p = _wt(wtype), _path(path)
    m, k = x.shape
    ptrs = [d if isinstance(d, int) else d.data_ptr() for d in destinations]
    arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
    ws = _workspace(compute_workspace_size(wt, m, n, k, p), x.device, workspace)
    nbytes = 0 if ws is None else ws.numel()
    _check(lib().pfng_b200_compute_gather(wt, _ptr(w), _ptr(x), x.stride(0), arr, len(ptrs), ldd, m, n, k,
                                          _ptr(ws), nbytes, p, _stream(stream)), "compute_gather")


def mm_gather(wtype, w, a, m: int, n: int, k: int, destinations, ldd: int, path="auto", workspace=None,
              stream=None) -> None:
    """compute_gather with pre-quantized activations `a` (q8_0 or q8_K bytes, as mm())."""
    wt, p = _wt(wtype), _path(path)
    ptrs = [d if isinstance(d, int) else d.data_ptr() for d in destinations]
    arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
    ws = _workspace(mm_workspace_size(wt, m, n, k, p), a.device, workspace)
    nbytes = 0 if ws is None else ws.numel()
    _check(lib().pfng_b200_mm_gather(wt, _ptr(w), _ptr(a), arr, len(ptrs), ldd, m, n, k, _ptr(ws), nbytes, p,
                                     _stream(stream)), "mm_gather")


def ipc_alloc(nbytes: int) -> tuple[int, bytes]:
    """A device buffer of the current GPU that other processes can open: (pointer, 64-byte handle)."""
    ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(lib().pfng_b200_ipc_alloc(nbytes, ctypes.byref(ptr), handle), "ipc_alloc")
    return ptr.value, handle.raw


def ipc_free(ptr: int) -> None:
    _check(lib().pfng_b200_ipc_free(ptr), "ipc_free")


def ipc_open(handle: bytes) -> int:
    """Device pointer (on the current GPU's address space) to another process's ipc_alloc buffer."""
    ptr = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES)
    _check(lib().pfng_b200_ipc_open(buf, ctypes.byref(ptr)), "ipc_open")
    return ptr.value


def ipc_close(ptr: int) -> None:
    _check(lib().pfng_b200_ipc_close(ptr), "ipc_close")


class _DeviceArray:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_tensor(ptr: int, shape, device=None):
    """A float32 torch tensor viewing `shape` floats at device pointer `ptr` (no copy, not owning)."""
    import torch
    return torch.as_tensor(_DeviceArray(ptr, shape, "<f4"), device=device or torch.device("cuda"))


class _Ipc:
    alloc = staticmethod(ipc_alloc)
    free = staticmethod(ipc_free)
    open = staticmethod(ipc_open)
    close = staticmethod(ipc_close)


class GatheredC:
    """Full fp32 C [m][n] on every rank of one node, writable by every rank.

    Each rank allocates its C with ipc_alloc; the handles are all-gathered
    over `group` (torch.distributed) and every rank opens the others'.  A rank
    whose weight rows are [begin, end) (shard_rows) passes
    destinations(begin) to compute_gather: its own C first, then the other
    ranks' C in rank order, each offset by `begin` columns, with ldd = n.
    `ipc` replaces the CUDA IPC calls (tests of the host logic)."""

    def __init__(self, m: int, n: int, group=None, ipc=None):
        import torch.distributed as dist
        self.m, self.n, self.group = m, n, group
        self._ipc = ipc or _Ipc
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.ptr, handle = self._ipc.alloc(max(1, m * n) * 4)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.bases = [self.ptr if r == self.rank else self._ipc.open(handles[r]) for r in range(self.world)]

    def destinations(self, col: int) -> list[int]:
        order = [self.rank] + [r for r in range(self.world) if r != self.rank]
        return [self.bases[r] + 4 * col for r in order]

    def tensor(self):
        """This rank's C as a torch tensor (valid until close())."""
        return device_tensor(self.ptr, (self.m, self.n))

    def close(self) -> None:
        """Unmap the other ranks' C, wait for every rank to do the same, free this rank's C."""
        import torch.distributed as dist
        if self.bases is None:
            return
        for r, b in enumerate(self.bases):
            if r != self.rank:
                self._ipc.close(b)
        dist.barrier(group=self.group)
        self._ipc.free(self.ptr)
        self.bases = None


def loaded_library_path() -> str:
    """Path of the shared object this process loaded (for provenance checks)."""
    lib()
    return os.path.realpath(LIB_PATH)
