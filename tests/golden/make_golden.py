"""Generate the golden fixtures in this directory from the reference itself.

Run in a checkout where the reference was compiled into oracle/_ref
(``make -C oracle``):

    python tests/golden/make_golden.py

Every expected value here is an output of the reference's own code
(bench/llama_reference/llama_reference.cpp and bench/framework/benchmark.cpp,
compiled in place by oracle/Makefile), never of this project's oracle or
kernels.  The fixtures pin the C restatement in oracle/ (tests/test_oracle.py)
and travel with the repository, so the pin holds where the reference is absent.

Cases:
  * ref_<type>_seed<s>: the reference's own seeded generator (create_input:
    U(-1, 1) activations/weights from std::mt19937, iq2_xxs grid indices 0..31),
    with the reference's quantized activations and its compute() output;
  * normal_<type>: N(0, 1) data (the distribution of the B200 benchmark
    configurations) quantized by the reference's quantizers, and its output;
  * quant_edges: quantizer inputs chosen for ties, zeros, subnormal scales and
    rounding boundaries, with the reference's block bytes;
  * fp16_edges: fp32 -> fp16 conversions of boundary values.
"""
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from oracle_lib import Reference, TYPES  # noqa: E402


def edge_rows(k: int) -> np.ndarray:
    rows = []
    rows.append(np.zeros(k, np.float32))                                   # all zero
    r = np.zeros(k, np.float32); r[5] = 1.0; rows.append(r)                # single value
    r = np.tile(np.array([0.5, -0.5], np.float32), k // 2); rows.append(r)  # equal-magnitude tie, + first
    r = np.tile(np.array([-0.5, 0.5], np.float32), k // 2); rows.append(r)  # equal-magnitude tie, - first
    r = (np.arange(k, dtype=np.float32) - k / 2) / (k / 2) * 127.0; rows.append(r)  # ramp
    r = np.full(k, 1e-30, np.float32); r[::3] = -3e-41; rows.append(r)     # subnormal scales
    r = (np.arange(k, dtype=np.float32) % 32 - 15.5) * 0.25; rows.append(r)  # .5 boundaries
    r = np.full(k, 65504.0 * 127.0, np.float32); r[1::2] *= -1; rows.append(r)  # fp16 overflow of d
    rng = np.random.default_rng(7)
    rows.append((rng.standard_normal(k) * 1e-3).astype(np.float32))
    rows.append((rng.standard_normal(k) * 1e3).astype(np.float32))
    return np.stack(rows)


def main() -> None:
    ref = Reference()
    out = {}
    shapes = {"q4_0": (3, 5, 256), "q4_K": (2, 3, 512), "iq2_xxs": (2, 3, 512)}
    for wtype, (m, n, k) in shapes.items():
        for seed in (1, 2):
            w, x = ref.create_input(wtype, m, n, k, seed)
            akind = "q8_0" if wtype == "q4_0" else "q8_K"
            a = ref.quantize(akind, x)
            c = ref.compute(wtype, w, x, m, n, k)
            key = f"ref_{wtype}_seed{seed}"
            out[f"{key}_w"] = w.view(np.uint8).reshape(-1)
            out[f"{key}_x"] = x
            out[f"{key}_a"] = a.view(np.uint8).reshape(-1)
            out[f"{key}_c"] = c
            out[f"{key}_shape"] = np.array([m, n, k], np.int64)
    rng = np.random.default_rng(20261201)
    for wtype, (m, n, k) in {"q4_0": (4, 6, 512), "q4_K": (3, 4, 768)}.items():
        wf = rng.standard_normal((n, k)).astype(np.float32)
        x = rng.standard_normal((m, k)).astype(np.float32)
        w = ref.quantize(wtype, wf)
        c = ref.compute(wtype, w, x, m, n, k)
        key = f"normal_{wtype}"
        out[f"{key}_wf"] = wf
        out[f"{key}_w"] = w.view(np.uint8).reshape(-1)
        out[f"{key}_x"] = x
        out[f"{key}_c"] = c
        out[f"{key}_shape"] = np.array([m, n, k], np.int64)
    e = edge_rows(256)
    for kind in ("q4_0", "q8_0", "q8_K", "q4_K"):
        out[f"quant_edges_{kind}"] = ref.quantize(kind, e).view(np.uint8).reshape(-1)
    out["quant_edges_x"] = e
    special = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.996, 65520.0, 65536.0, 1e9, -1e9,
                        6.1035156e-05, 6.1035153e-05, 5.9604645e-08, 2.9802322e-08, 2.9802326e-08,
                        8.940697e-08, 1.0009765625, 1.00048828125, 1.00146484375, np.inf, -np.inf,
                        1.0 / 127.0, 3.0 / 127.0, 1e-40, -1e-45], np.float32)
    out["fp16_edges_x"] = special
    out["fp16_edges_h"] = ref.fp32_to_fp16(special)
    np.savez_compressed(HERE / "golden.npz", **out)
    print("wrote", HERE / "golden.npz", sum(v.nbytes for v in out.values()), "bytes uncompressed")


if __name__ == "__main__":
    main()
