"""ctypes access to the parity checkers (test infrastructure).

* `Oracle` wraps oracle/liboracle.so, the C restatement of the reference's
  scalar ggml path (oracle/pfng_oracle.c).
* `Reference` wraps oracle/_ref/libpfng_ref.so, the reference's own
  llama_reference / benchmark sources compiled in place (oracle/Makefile).
  It exists only where the reference checkout was present at build time.

Both work on numpy arrays; block arrays are numpy structured dtypes with the
ggml wire layout (include/ggml.h:125-159 of the reference).
"""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent.parent
ORACLE_SO = ROOT / "oracle" / "liboracle.so"
REF_SO = ROOT / "oracle" / "_ref" / "libpfng_ref.so"
REF_TABLES_SO = ROOT / "oracle" / "_ref" / "libpfng_ref_tables.so"

BLOCK_Q4_0 = np.dtype([("d", "<u2"), ("qs", "u1", 16)])
BLOCK_Q8_0 = np.dtype([("d", "<u2"), ("qs", "i1", 32)])
BLOCK_Q8_K = np.dtype([("d", "<f4"), ("qs", "i1", 256), ("bsums", "<i2", 16)])
BLOCK_IQ2_XXS = np.dtype([("d", "<u2"), ("qs", "<u2", 32)])
BLOCK_Q4_K = np.dtype([("d", "<u2"), ("dmin", "<u2"), ("scales", "u1", 12), ("qs", "u1", 128)])
assert BLOCK_Q4_0.itemsize == 18 and BLOCK_Q8_0.itemsize == 34 and BLOCK_Q8_K.itemsize == 292
assert BLOCK_IQ2_XXS.itemsize == 66 and BLOCK_Q4_K.itemsize == 144

# weight type -> (weight block dtype, weight block K, activation block dtype, activation block K)
TYPES = {
    "q4_0": (BLOCK_Q4_0, 32, BLOCK_Q8_0, 32),
    "q4_K": (BLOCK_Q4_K, 256, BLOCK_Q8_K, 256),
    "iq2_xxs": (BLOCK_IQ2_XXS, 256, BLOCK_Q8_K, 256),
}
TYPE_INDEX = {"q4_0": 0, "q4_K": 1, "iq2_xxs": 2}

_P = ctypes.c_void_p
_S = ctypes.c_size_t


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class Oracle:
    def __init__(self, path: pathlib.Path = ORACLE_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (run make -C oracle)")
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.oracle_fp16_to_fp32.restype = ctypes.c_float
        L.oracle_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.oracle_fp32_to_fp16.restype = ctypes.c_uint16
        L.oracle_fp32_to_fp16.argtypes = [ctypes.c_float]
        for name in ("q4_0", "q8_0", "q8_K", "q4_K"):
            f = getattr(L, f"oracle_quantize_{name}")
            f.restype = None
            f.argtypes = [_P, _P, _S, _S]
        for t in ("q4_0_q8_0", "q4_K_q8_K", "iq2_xxs_q8_K"):
            f = getattr(L, f"oracle_mm_{t}")
            f.restype = None
            f.argtypes = [_P, _P, _P, _S, _S, _S, _S]
            f = getattr(L, f"oracle_partials_{t}")
            f.restype = None
            f.argtypes = [_P, _P, _P, _S, _S, _S]
            f = getattr(L, f"oracle_bound_{t}")
            f.restype = None
            f.argtypes = [_P, _P, _P, _S, _S, _S]
        for t in ("q4_0", "q4_K", "iq2_xxs"):
            f = getattr(L, f"oracle_compute_{t}")
            f.restype = None
            f.argtypes = [_P, _P, _P, _S, _S, _S]
        for name in ("pack", "unpack"):
            f = getattr(L, f"oracle_{name}_q4_0_planar")
            f.restype = None
            f.argtypes = [_P, _P, _S, _S]
        L.oracle_iq2_xxs_grid.restype = ctypes.c_uint64
        L.oracle_iq2_xxs_grid.argtypes = [ctypes.c_uint]
        L.oracle_iq2_xxs_sign_mask.restype = ctypes.c_uint8
        L.oracle_iq2_xxs_sign_mask.argtypes = [ctypes.c_uint]
        L.oracle_iq2_xxs_decode_group.restype = None
        L.oracle_iq2_xxs_decode_group.argtypes = [_P, _P, _P]

    # -- codecs
    def fp32_to_fp16(self, x: np.ndarray) -> np.ndarray:
        f = self.lib.oracle_fp32_to_fp16
        return np.array([f(float(v)) for v in np.asarray(x, np.float32).ravel()], np.uint16)

    # -- quantizers: x is (m, k) float32
    def quantize(self, kind: str, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        m, k = x.shape
        dtype, qk = {"q4_0": (BLOCK_Q4_0, 32), "q8_0": (BLOCK_Q8_0, 32),
                     "q8_K": (BLOCK_Q8_K, 256), "q4_K": (BLOCK_Q4_K, 256)}[kind]
        y = np.zeros((m, k // qk), dtype)
        getattr(self.lib, f"oracle_quantize_{kind}")(ptr(x), ptr(y), m, k)
        return y

    @staticmethod
    def _suffix(wtype: str) -> str:
        return {"q4_0": "q4_0_q8_0", "q4_K": "q4_K_q8_K", "iq2_xxs": "iq2_xxs_q8_K"}[wtype]

    def mm(self, wtype: str, w: np.ndarray, a: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        c = np.zeros((m, n), np.float32)
        getattr(self.lib, f"oracle_mm_{self._suffix(wtype)}")(ptr(w), ptr(a), ptr(c), m, n, k, n)
        return c

    def compute(self, wtype: str, w: np.ndarray, x: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        c = np.zeros((m, n), np.float32)
        getattr(self.lib, f"oracle_compute_{wtype}")(ptr(w), ptr(x), ptr(c), m, n, k)
        return c

    def partials(self, wtype: str, w: np.ndarray, a: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        out = np.zeros((m, n, k // 32), np.int32)
        getattr(self.lib, f"oracle_partials_{self._suffix(wtype)}")(ptr(w), ptr(a), ptr(out), m, n, k)
        return out

    def bound(self, wtype: str, w: np.ndarray, a: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        out = np.zeros((m, n), np.float64)
        getattr(self.lib, f"oracle_bound_{self._suffix(wtype)}")(ptr(w), ptr(a), ptr(out), m, n, k)
        return out

    # -- q4_0 planar row layout: w is (n, k / 32) block_q4_0, the result raw bytes (n, 18 k / 32)
    def pack_q4_0_planar(self, w: np.ndarray, n: int, k: int) -> np.ndarray:
        w = np.ascontiguousarray(w)
        out = np.zeros((n, k // 32 * 18), np.uint8)
        self.lib.oracle_pack_q4_0_planar(ptr(w), ptr(out), n, k)
        return out

    def unpack_q4_0_planar(self, wp: np.ndarray, n: int, k: int) -> np.ndarray:
        wp = np.ascontiguousarray(wp, np.uint8)
        out = np.zeros((n, k // 32), BLOCK_Q4_0)
        self.lib.oracle_unpack_q4_0_planar(ptr(wp), ptr(out), n, k)
        return out

    def iq2_grid(self) -> np.ndarray:
        return np.array([self.lib.oracle_iq2_xxs_grid(i) for i in range(256)], np.uint64)

    def iq2_sign_mask(self) -> np.ndarray:
        return np.array([self.lib.oracle_iq2_xxs_sign_mask(i) for i in range(128)], np.uint8)

    def iq2_decode_group(self, packed8: np.ndarray) -> tuple[np.ndarray, int]:
        packed8 = np.ascontiguousarray(packed8, np.uint8)
        values = np.zeros(32, np.int8)
        scale = ctypes.c_int(0)
        self.lib.oracle_iq2_xxs_decode_group(ptr(packed8), ptr(values), ctypes.addressof(scale))
        return values, scale.value


class Reference:
    """The reference's own code (oracle/_ref), for pinning and golden vectors."""

    def __init__(self, path: pathlib.Path = REF_SO, tables: pathlib.Path = REF_TABLES_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (reference checkout absent at build time)")
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.ref_fp32_to_fp16_array.restype = None
        L.ref_fp32_to_fp16_array.argtypes = [_P, _P, _S]
        L.ref_fp16_to_fp32_array.restype = None
        L.ref_fp16_to_fp32_array.argtypes = [_P, _P, _S]
        for name in ("q4_0", "q8_0", "q8_K", "q4_K"):
            f = getattr(L, f"ref_quantize_{name}")
            f.restype = None
            f.argtypes = [_P, _P, _S, _S]
        L.ref_compute.restype = ctypes.c_int
        L.ref_compute.argtypes = [ctypes.c_int, _P, _P, _P, _S, _S, _S]
        L.ref_mm_threads.restype = ctypes.c_int
        L.ref_mm_threads.argtypes = [ctypes.c_int, _P, _P, _P, _S, _S, _S, _S, ctypes.c_int]
        L.ref_create_input.restype = ctypes.c_int
        L.ref_create_input.argtypes = [ctypes.c_int, _S, _S, _S, ctypes.c_uint64, _P, _P]
        L.ref_iq2_decode_subblock.restype = None
        L.ref_iq2_decode_subblock.argtypes = [_P, _P, _P]
        self.tables = ctypes.CDLL(str(tables)) if tables.exists() else None
        if self.tables is not None:
            self.tables.ref_iq2xxs_grid_upstream.restype = ctypes.c_uint64
            self.tables.ref_iq2xxs_grid_upstream.argtypes = [ctypes.c_uint]
            self.tables.ref_keven_signs_q2xs.restype = ctypes.c_int
            self.tables.ref_keven_signs_q2xs.argtypes = [ctypes.c_uint]
            self.tables.ref_ksigns_iq2xs.restype = ctypes.c_uint8
            self.tables.ref_ksigns_iq2xs.argtypes = [ctypes.c_uint]

    def fp32_to_fp16(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.shape, np.uint16)
        self.lib.ref_fp32_to_fp16_array(ptr(x), ptr(out), x.size)
        return out

    def fp16_to_fp32(self, h: np.ndarray) -> np.ndarray:
        h = np.ascontiguousarray(h, np.uint16)
        out = np.zeros(h.shape, np.float32)
        self.lib.ref_fp16_to_fp32_array(ptr(h), ptr(out), h.size)
        return out

    def quantize(self, kind: str, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        m, k = x.shape
        dtype, qk = {"q4_0": (BLOCK_Q4_0, 32), "q8_0": (BLOCK_Q8_0, 32),
                     "q8_K": (BLOCK_Q8_K, 256), "q4_K": (BLOCK_Q4_K, 256)}[kind]
        y = np.zeros((m, k // qk), dtype)
        getattr(self.lib, f"ref_quantize_{kind}")(ptr(x), ptr(y), m, k)
        return y

    def compute(self, wtype: str, w: np.ndarray, x: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        c = np.zeros((m, n), np.float32)
        assert self.lib.ref_compute(TYPE_INDEX[wtype], ptr(w), ptr(x), ptr(c), m, n, k) == 0
        return c

    def mm_threads(self, wtype: str, w: np.ndarray, a: np.ndarray, m: int, n: int, k: int, threads: int) -> np.ndarray:
        c = np.zeros((m, n), np.float32)
        assert self.lib.ref_mm_threads(TYPE_INDEX[wtype], ptr(w), ptr(a), ptr(c), m, n, k, n, threads) == 0
        return c

    def create_input(self, wtype: str, m: int, n: int, k: int, seed: int = 1):
        wdt, wqk, _, _ = TYPES[wtype]
        x = np.zeros((m, k), np.float32)
        w = np.zeros((n, k // wqk), wdt)
        assert self.lib.ref_create_input(TYPE_INDEX[wtype], m, n, k, seed, ptr(x), ptr(w)) == 0
        return w, x

    def iq2_decode_subblock(self, packed8: np.ndarray) -> tuple[np.ndarray, int]:
        packed8 = np.ascontiguousarray(packed8, np.uint8)
        values = np.zeros(32, np.int8)
        scale = ctypes.c_int(0)
        self.lib.ref_iq2_decode_subblock(ptr(packed8), ptr(values), ctypes.addressof(scale))
        return values, scale.value


def reference_or_none() -> Reference | None:
    try:
        return Reference()
    except FileNotFoundError:
        return None
