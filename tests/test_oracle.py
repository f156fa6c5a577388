"""The oracle (oracle/pfng_oracle.c) against the reference's own outputs.

The golden fixtures were produced by the reference's code
(tests/golden/make_golden.py); where the reference is compiled here
(oracle/_ref) it is also compared directly on fresh random inputs.
"""
import numpy as np
import pytest

from oracle_lib import BLOCK_Q8_0, BLOCK_Q8_K, TYPES


def test_oracle_matches_golden_compute(oracle, golden):
    for wtype in TYPES:
        wdt, wqk, adt, aqk = TYPES[wtype]
        for seed in (1, 2):
            key = f"ref_{wtype}_seed{seed}"
            m, n, k = (int(v) for v in golden[f"{key}_shape"])
            w = golden[f"{key}_w"].view(wdt)
            x = golden[f"{key}_x"]
            c = oracle.compute(wtype, w, x, m, n, k)
            np.testing.assert_array_equal(c.view(np.uint32), golden[f"{key}_c"].view(np.uint32), err_msg=key)
            a = oracle.quantize("q8_0" if wtype == "q4_0" else "q8_K", x)
            assert a.tobytes() == golden[f"{key}_a"].tobytes(), key


def test_oracle_matches_golden_normal(oracle, golden):
    for wtype in ("q4_0", "q4_K"):
        key = f"normal_{wtype}"
        m, n, k = (int(v) for v in golden[f"{key}_shape"])
        w = oracle.quantize(wtype, golden[f"{key}_wf"])
        assert w.tobytes() == golden[f"{key}_w"].tobytes(), key
        c = oracle.compute(wtype, w, golden[f"{key}_x"], m, n, k)
        np.testing.assert_array_equal(c.view(np.uint32), golden[f"{key}_c"].view(np.uint32))


def test_oracle_quantizer_edges(oracle, golden):
    x = golden["quant_edges_x"]
    for kind in ("q4_0", "q8_0", "q8_K", "q4_K"):
        assert oracle.quantize(kind, x).tobytes() == golden[f"quant_edges_{kind}"].tobytes(), kind


def test_oracle_fp16_edges(oracle, golden):
    np.testing.assert_array_equal(oracle.fp32_to_fp16(golden["fp16_edges_x"]), golden["fp16_edges_h"])


def test_oracle_fp16_matches_ieee_rne(oracle):
    # ggml's conversion (ggml.h:99-117) is IEEE round-to-nearest-even for
    # every non-NaN input; numpy's float16 cast is too.
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2**32, size=20000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[~np.isnan(x)]
    with np.errstate(over="ignore"):
        expect = x.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(oracle.fp32_to_fp16(x), expect)


def test_oracle_partials_fold_to_mm(oracle):
    # sum_b isum_b * dw_b * da_b in block order reproduces the q4_0 dot exactly
    rng = np.random.default_rng(11)
    m, n, k = 2, 3, 256
    w = oracle.quantize("q4_0", rng.standard_normal((n, k)).astype(np.float32))
    a = oracle.quantize("q8_0", rng.standard_normal((m, k)).astype(np.float32))
    p = oracle.partials("q4_0", w, a, m, n, k)
    c = oracle.mm("q4_0", w, a, m, n, k)
    dw = w["d"].view(np.float16).astype(np.float32)
    da = a["d"].view(np.float16).astype(np.float32)
    for i in range(m):
        for j in range(n):
            s = np.float32(0)
            for b in range(k // 32):
                s = np.float32(s + np.float32(np.float32(p[i, j, b]) * dw[j, b]) * da[i, b])
            assert s == c[i, j]


def test_oracle_bound_dominates_error(oracle):
    rng = np.random.default_rng(5)
    m, n, k = 3, 4, 512
    for wtype in TYPES:
        if wtype == "iq2_xxs":
            continue
        w = oracle.quantize(wtype, rng.standard_normal((n, k)).astype(np.float32))
        a = oracle.quantize("q8_0" if wtype == "q4_0" else "q8_K", rng.standard_normal((m, k)).astype(np.float32))
        c = oracle.mm(wtype, w, a, m, n, k)
        bound = oracle.bound(wtype, w, a, m, n, k)
        assert np.all(bound >= np.abs(c) * (1 - 1e-6))


def test_iq2_sign_mask_matches_ksigns(oracle, reference):
    if reference.tables is None:
        pytest.skip("reference table shim not built")
    ours = oracle.iq2_sign_mask()
    theirs = np.array([reference.tables.ref_ksigns_iq2xs(i) for i in range(128)], np.uint8)
    np.testing.assert_array_equal(ours, theirs)
    # and the even-sign table: bit l of mask i <-> keven_signs_q2xs[8 i + l] == -1
    even = np.array([reference.tables.ref_keven_signs_q2xs(i) for i in range(1024)]).reshape(128, 8)
    bits = (ours[:, None] >> np.arange(8)) & 1
    np.testing.assert_array_equal(bits == 1, even == -1)


def test_iq2_grid_matches_reference_tables(oracle, reference):
    if reference.tables is None:
        pytest.skip("reference table shim not built")
    ours = oracle.iq2_grid()
    theirs = np.array([reference.tables.ref_iq2xxs_grid_upstream(i) for i in range(256)], np.uint64)
    np.testing.assert_array_equal(ours, theirs)


def test_iq2_decode_matches_reference_subset(oracle, reference):
    rng = np.random.default_rng(9)
    for _ in range(200):
        packed = rng.integers(0, 256, 8).astype(np.uint8)
        packed[:4] %= 32  # the reference's decoder holds the first 32 grid points
        v1, s1 = oracle.iq2_decode_group(packed)
        v2, s2 = reference.iq2_decode_subblock(packed)
        np.testing.assert_array_equal(v1, v2)
        assert s1 == s2


@pytest.mark.parametrize("wtype", list(TYPES))
def test_oracle_matches_reference_random(oracle, reference, wtype):
    rng = np.random.default_rng(17)
    m, n, k = 3, 7, 1024
    if wtype == "iq2_xxs":
        w, x = reference.create_input(wtype, m, n, k, seed=5)
    else:
        wf = rng.standard_normal((n, k)).astype(np.float32)
        w = reference.quantize(wtype, wf)
        assert oracle.quantize(wtype, wf).tobytes() == w.tobytes()
        x = rng.standard_normal((m, k)).astype(np.float32)
    c1 = oracle.compute(wtype, w, x, m, n, k)
    c2 = reference.compute(wtype, w, x, m, n, k)
    np.testing.assert_array_equal(c1.view(np.uint32), c2.view(np.uint32))


def test_reference_threaded_matches_compute(reference):
    rng = np.random.default_rng(2)
    m, n, k = 4, 9, 512
    for wtype in TYPES:
        w, x = reference.create_input(wtype, m, n, k, seed=3)
        a = reference.quantize("q8_0" if wtype == "q4_0" else "q8_K", x)
        c1 = reference.mm_threads(wtype, w, a, m, n, k, threads=3)
        c2 = reference.compute(wtype, w, x, m, n, k)
        np.testing.assert_array_equal(c1.view(np.uint32), c2.view(np.uint32))


def test_planar_layout_oracle(oracle, golden):
    # the planar row layout is a per-row byte permutation of block_q4_0:
    # nibble fields first (16 B per block), then the fp16 scales; checked on
    # the reference generator's q4_0 weights (golden fixture) and on random bytes
    import numpy as np
    m, n, k = (int(v) for v in golden["ref_q4_0_seed1_shape"])
    rng = np.random.default_rng(3)
    for w, n, k in ((golden["ref_q4_0_seed1_w"], n, k),
                    (rng.integers(0, 256, 7 * 48 * 18, dtype=np.uint8), 7, 1536)):
        nb = k // 32
        blocks = w.reshape(n, nb, 18)
        planar = oracle.pack_q4_0_planar(w, n, k)
        assert planar.shape == (n, nb * 18)
        np.testing.assert_array_equal(planar[:, : 16 * nb].reshape(n, nb, 16), blocks[:, :, 2:])
        np.testing.assert_array_equal(planar[:, 16 * nb:].reshape(n, nb, 2), blocks[:, :, :2])
        assert oracle.unpack_q4_0_planar(planar, n, k).tobytes() == w.tobytes()
