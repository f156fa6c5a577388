"""Parity of the B200 kernels with the reference's scalar path (GPU).

Every call goes through the C ABI (libpfng_b200.so via pfng_b200).  The bar:
  * quantizer bytes and integer per-32 partial dot products: bit-exact;
  * fp32 outputs: |C - C_ref| <= 1e-5 * sum_k |w_k a_k| per element, where
    C_ref is the oracle's (the reference's) result on the same quantized
    inputs and the bound is computed by the oracle;
  * the SIMPLE path restates the reference operation for operation and must
    be bit-identical.
"""
import numpy as np
import pytest

from oracle_lib import BLOCK_Q8_0, BLOCK_Q8_K, TYPES

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import pfng_b200 as pb  # noqa: E402

TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    yield
    pb.check_kernel_error()


def dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dev_bytes(blocks: np.ndarray):
    return dev(blocks.view(np.uint8).reshape(-1))


def host(t) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def act_kind(wtype):
    return "q8_0" if wtype == "q4_0" else "q8_K"


def make_weights(oracle, wtype, n, k, rng, full_range=True):
    wdt = TYPES[wtype][0]
    if wtype == "iq2_xxs":
        w = np.zeros((n, k // 256), wdt)
        w["d"] = rng.uniform(1e-3, 1e-2, size=w.shape).astype(np.float16).view(np.uint16)
        qs = w["qs"].view(np.uint8).reshape(n, k // 256, 8, 8)
        qs[..., :4] = rng.integers(0, 256 if full_range else 32, size=qs[..., :4].shape)
        qs[..., 4:] = rng.integers(0, 256, size=qs[..., 4:].shape)
        return w
    return oracle.quantize(wtype, rng.standard_normal((n, k)).astype(np.float32))


def check_close(c, ref, bound, what):
    err = np.abs(c.astype(np.float64) - ref.astype(np.float64))
    limit = TOL * bound + 1e-30
    bad = ~(err <= limit)  # NaN fails too
    assert not bad.any(), f"{what}: {bad.sum()} elements out of tolerance, worst {np.max(err / limit):.3g}x"


# --------------------------------------------------------------- quantizers
def quant_inputs(k):
    rng = np.random.default_rng(1)
    rows = [rng.standard_normal((19, k)), rng.uniform(-1, 1, (7, k)), rng.standard_normal((3, k)) * 1e-3,
            rng.standard_normal((3, k)) * 1e3, np.zeros((1, k)),
            np.tile(np.array([0.5, -0.5]), (1, k // 2)), np.tile(np.array([-0.25, 0.25]), (1, k // 2))]
    return np.concatenate(rows).astype(np.float32)


@pytest.mark.parametrize("kind", ["q8_0", "q8_K", "q4_0", "q4_K"])
@pytest.mark.parametrize("pad", [0, 1, 4])
def test_quantizer_bitexact(oracle, kind, pad):
    k = 1024
    x = quant_inputs(k)
    xp = np.zeros((x.shape[0], k + pad), np.float32)
    xp[:, :k] = x
    xd = dev(xp)[:, :k]
    fn = {"q8_0": pb.quantize_q8_0, "q8_K": pb.quantize_q8_K, "q4_0": pb.quantize_q4_0, "q4_K": pb.quantize_q4_K}[kind]
    got = host(fn(xd))
    assert got.tobytes() == oracle.quantize(kind, x).tobytes()


def test_quantizer_golden_edges(golden):
    x = golden["quant_edges_x"]
    xd = dev(x)
    for kind, fn in (("q8_0", pb.quantize_q8_0), ("q8_K", pb.quantize_q8_K), ("q4_0", pb.quantize_q4_0),
                     ("q4_K", pb.quantize_q4_K)):
        assert host(fn(xd)).tobytes() == golden[f"quant_edges_{kind}"].tobytes(), kind


def test_weight_quantizer_full_size(oracle):
    rng = np.random.default_rng(4)
    wf = (rng.standard_normal((4096, 4096)) * 0.02).astype(np.float32)
    wd = dev(wf)
    assert host(pb.quantize_q4_0(wd)).tobytes() == oracle.quantize("q4_0", wf).tobytes()
    assert host(pb.quantize_q4_K(wd[:1024])).tobytes() == oracle.quantize("q4_K", wf[:1024]).tobytes()


# ------------------------------------------------------------------- matmul
CASES = [
    # (wtype, path, m, n, k)
    ("q4_0", "gemv", 1, 300, 1024), ("q4_0", "gemv", 3, 257, 2048), ("q4_0", "gemv", 8, 64, 4096),
    ("q4_0", "mma", 9, 129, 256), ("q4_0", "mma", 130, 300, 1536), ("q4_0", "mma", 256, 256, 1024),
    ("q4_0", "simple", 5, 17, 96), ("q4_0", "simple", 33, 40, 512),
    ("q4_K", "gemv", 1, 300, 1536), ("q4_K", "gemv", 5, 100, 2048), ("q4_K", "mma", 9, 129, 256),
    ("q4_K", "mma", 140, 260, 1536), ("q4_K", "simple", 6, 21, 512),
    ("iq2_xxs", "gemv", 1, 304, 1536), ("iq2_xxs", "gemv", 7, 64, 2048), ("iq2_xxs", "mma", 9, 129, 256),
    ("iq2_xxs", "mma", 140, 264, 1536), ("iq2_xxs", "simple", 4, 19, 512),
]


@pytest.mark.parametrize("wtype,path,m,n,k", CASES)
def test_mm_parity(oracle, wtype, path, m, n, k):
    rng = np.random.default_rng(m * 1000 + n + k)
    w = make_weights(oracle, wtype, n, k, rng)
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = oracle.quantize(act_kind(wtype), x)
    ref = oracle.mm(wtype, w, a, m, n, k)
    bound = oracle.bound(wtype, w, a, m, n, k)
    wd, ad = dev_bytes(w), dev_bytes(a)
    c = host(pb.mm(wtype, wd, ad, m, n, k, path=path))
    if path == "simple":
        np.testing.assert_array_equal(c.view(np.uint32), ref.view(np.uint32))
    else:
        check_close(c, ref, bound, f"{wtype}/{path}/{m}x{n}x{k}")
    # the fused fp32 entry gives the same bits as mm on the quantized rows
    c2 = host(pb.compute(wtype, wd, dev(x), n, path=path))
    np.testing.assert_array_equal(c2.view(np.uint32), c.view(np.uint32))


@pytest.mark.parametrize("wtype,path,m,n,k", [c for c in CASES if c[1] != "simple" or c[4] >= 256])
def test_partials_bitexact(oracle, wtype, path, m, n, k):
    rng = np.random.default_rng(m + n * 7 + k)
    w = make_weights(oracle, wtype, n, k, rng)
    a = oracle.quantize(act_kind(wtype), rng.standard_normal((m, k)).astype(np.float32))
    got = host(pb.partials(wtype, dev_bytes(w), dev_bytes(a), m, n, k, path=path))
    np.testing.assert_array_equal(got, oracle.partials(wtype, w, a, m, n, k))


@pytest.mark.parametrize("wtype", list(TYPES))
def test_reference_generator_inputs(oracle, golden, wtype):
    # the reference's own seeded inputs (create_input, U(-1,1)) and outputs
    for seed in (1, 2):
        key = f"ref_{wtype}_seed{seed}"
        m, n, k = (int(v) for v in golden[f"{key}_shape"])
        wd = dev(golden[f"{key}_w"])
        x = golden[f"{key}_x"]
        ref = golden[f"{key}_c"]
        for path in ("auto", "simple"):
            c = host(pb.compute(wtype, wd, dev(x), n, path=path))
            if path == "simple":
                np.testing.assert_array_equal(c.view(np.uint32), ref.view(np.uint32))
            else:
                w = golden[f"{key}_w"].view(TYPES[wtype][0])
                a = oracle.quantize(act_kind(wtype), x)
                check_close(c, ref, oracle.bound(wtype, w, a, m, n, k), key)


def test_edge_shapes(oracle):
    rng = np.random.default_rng(0)
    w = make_weights(oracle, "q4_0", 8, 256, rng)
    wd = dev_bytes(w)
    # k == 0: C is all zeros
    c = torch.full((3, 8), float("nan"), device="cuda")
    pb.mm("q4_0", wd, wd, 3, 8, 0, out=c)
    assert torch.count_nonzero(c).item() == 0
    # m == 0 / n == 0: no-ops
    pb.mm("q4_0", wd, wd, 0, 8, 256, out=torch.empty((0, 8), device="cuda"))
    # ldc > n leaves the padding untouched
    x = rng.standard_normal((4, 256)).astype(np.float32)
    a = oracle.quantize("q8_0", x)
    for path, m in (("gemv", 4), ("mma", 4), ("simple", 4)):
        big = torch.full((m, 11), -7.0, device="cuda")
        pb.mm("q4_0", wd, dev_bytes(a), m, 8, 256, out=big[:, :8], path=path)
        hb = host(big)
        assert np.all(hb[:, 8:] == -7.0)
        check_close(hb[:, :8], oracle.mm("q4_0", w, a, m, 8, 256), oracle.bound("q4_0", w, a, m, 8, 256), path)


def test_forced_path_rejections():
    wd = torch.zeros(18 * 10 * 3, dtype=torch.uint8, device="cuda")
    ad = torch.zeros(34 * 16 * 3, dtype=torch.uint8, device="cuda")
    with pytest.raises(pb.PfngError) as e:
        pb.mm("q4_0", wd, ad, 16, 10, 96, path="gemv")  # m > 8
    assert e.value.status == -7
    with pytest.raises(pb.PfngError):
        pb.mm("q4_0", wd, ad, 16, 10, 96, path="mma")   # k not a multiple of 256


# Full-size BASELINE configurations: tests/test_gpu_configs.py (whole matrices against the reference).


def test_unshard_columns():
    m, n, world, granule = 5, 1000, 3, 128
    full = torch.randn(m, n, device="cuda")
    spans = [pb.shard_rows(n, world, r, granule) for r in range(world)]
    width = max(e - b for b, e in spans)
    slices = torch.zeros(world, m, width, device="cuda")
    for r, (b, e) in enumerate(spans):
        slices[r, :, : e - b] = full[:, b:e]
    out = pb.unshard_columns(slices, m, n, world, granule)
    assert torch.equal(out, full)


@pytest.mark.parametrize("wtype", list(TYPES))
@pytest.mark.parametrize("m", [1, 3])
def test_grouped_matches_single(oracle, wtype, m):
    # several weight matrices sharing one activation, one launch; each output
    # equals the single-matrix GEMV bit for bit and the oracle within tolerance
    rng = np.random.default_rng(31 + m)
    k = 1536 if wtype != "q4_0" else 1024
    ns = [300, 64, 1000] if wtype != "iq2_xxs" else [304, 64, 1000]
    ws = [make_weights(oracle, wtype, n, k, rng) for n in ns]
    x = rng.standard_normal((m, k)).astype(np.float32)
    wds = [dev_bytes(w) for w in ws]
    xd = dev(x)
    outs = pb.compute_grouped(wtype, wds, xd, ns)
    a = oracle.quantize(act_kind(wtype), x)
    for w, wd, n, o in zip(ws, wds, ns, outs):
        single = host(pb.compute(wtype, wd, xd, n, path="gemv"))
        got = host(o)
        np.testing.assert_array_equal(got.view(np.uint32), single.view(np.uint32))
        check_close(got, oracle.mm(wtype, w, a, m, n, k), oracle.bound(wtype, w, a, m, n, k), f"grouped {wtype}")


def test_grouped_rejects_large_m():
    w = torch.zeros(18 * 64 * 8, dtype=torch.uint8, device="cuda")
    x = torch.zeros((9, 256), device="cuda")
    with pytest.raises(pb.PfngError) as e:
        pb.compute_grouped("q4_0", [w], x, [64])
    assert e.value.status == -7


def test_grouped_overlap_keeps_order(oracle):
    # back-to-back launches with PFNG_B200_OVERLAP_WEIGHTS: each may start
    # streaming its weights early, but reads its activations and writes its
    # outputs after the preceding kernel -- here the activations of each call
    # are produced by the kernel just before it.
    rng = np.random.default_rng(44)
    k, ns = 4096, [4096, 1000]
    sets = [[make_weights(oracle, "q4_0", n, k, rng) for n in ns] for _ in range(3)]
    dsets = [[dev_bytes(w) for w in s] for s in sets]
    x0 = dev(rng.standard_normal((1, k)).astype(np.float32))
    outs = [torch.empty((1, n), device="cuda") for n in ns]
    expected = None
    xs = []
    x = x0
    for r in range(3):
        x = x * 1.5 + 0.25  # produced by a torch kernel right before the call
        xs.append(x)
        pb.compute_grouped("q4_0", dsets[r], x, ns, outs=outs, overlap_weights=True)
    got = [host(o) for o in outs]
    for g, n in enumerate(ns):
        single = host(pb.compute("q4_0", dsets[2][g], xs[2], n, path="gemv"))
        np.testing.assert_array_equal(got[g].view(np.uint32), single.view(np.uint32))


# ------------------------------------------------- tcgen05 / TMEM q4_0 kernel
@pytest.mark.parametrize("m,n,k", [(9, 129, 256), (130, 300, 1536), (64, 128, 512), (480, 1536, 1536),
                                   (1000, 520, 2048)])
def test_q4_0_tcgen05_kernel(oracle, monkeypatch, m, n, k):
    # The tensor-memory kernel (selected with PFNG_B200_GEMM=tc) against the
    # oracle within tolerance, and bit-identical to the mma.sync kernel: both
    # fold the same integer sub-block sums in the same order.
    rng = np.random.default_rng(m * 31 + n + k)
    w = oracle.quantize("q4_0", rng.standard_normal((n, k)).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = oracle.quantize("q8_0", x)
    ref = oracle.mm("q4_0", w, a, m, n, k)
    bound = oracle.bound("q4_0", w, a, m, n, k)
    wd, xd = dev_bytes(w), dev(x)
    monkeypatch.setenv("PFNG_B200_GEMM", "tc")
    c_tc = host(pb.compute("q4_0", wd, xd, n, path="mma"))
    pb.check_kernel_error()
    monkeypatch.setenv("PFNG_B200_GEMM", "mma")
    monkeypatch.setenv("PFNG_B200_GEMM_SPLITS", "1")  # same summation order as the tcgen05 kernel
    c_mma = host(pb.compute("q4_0", wd, xd, n, path="mma"))
    check_close(c_tc, ref, bound, f"tcgen05 q4_0 {m}x{n}x{k}")
    np.testing.assert_array_equal(c_tc.view(np.uint32), c_mma.view(np.uint32))


@pytest.mark.parametrize("wtype", ["q4_K", "iq2_xxs"])
@pytest.mark.parametrize("n,k", [(4096, 4096), (1000, 2048), (520, 1536)])
def test_k_types_decode(oracle, wtype, n, k):
    # m = 1 decode shapes of the K-block types (register paths for k <= 4096):
    # integer partials bit-exact, fp32 within tolerance, grouped == single
    rng = np.random.default_rng(n + k)
    w = make_weights(oracle, wtype, n, k, rng)
    x = rng.standard_normal((1, k)).astype(np.float32)
    a = oracle.quantize("q8_K", x)
    wd, xd = dev_bytes(w), dev(x)
    c = host(pb.compute(wtype, wd, xd, n, path="gemv"))
    check_close(c, oracle.mm(wtype, w, a, 1, n, k), oracle.bound(wtype, w, a, 1, n, k), f"{wtype} decode {n}x{k}")
    got = host(pb.partials(wtype, wd, dev_bytes(a), 1, n, k, path="gemv"))
    np.testing.assert_array_equal(got, oracle.partials(wtype, w, a, 1, n, k))
    g = host(pb.compute_grouped(wtype, [wd], xd, [n])[0])
    np.testing.assert_array_equal(g.view(np.uint32), c.view(np.uint32))


@pytest.mark.parametrize("m,n,k", [(32, 4096, 4096), (17, 1000, 2048), (32, 4096, 11008), (64, 640, 4096)])
def test_split_k_small_m(oracle, monkeypatch, m, n, k):
    # small-m GEMM shapes whose tiles leave SMs idle run split-K: the splits'
    # fp32 tiles are added in split order -- within tolerance of the oracle,
    # deterministic, and every output format converts the same reduced C
    rng = np.random.default_rng(m + n + k)
    w = oracle.quantize("q4_0", rng.standard_normal((n, k)).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = oracle.quantize("q8_0", x)
    wd, xd = dev_bytes(w), dev(x)
    c = host(pb.compute("q4_0", wd, xd, n, path="mma"))
    check_close(c, oracle.mm("q4_0", w, a, m, n, k), oracle.bound("q4_0", w, a, m, n, k), f"split-K {m}x{n}x{k}")
    c2 = host(pb.compute("q4_0", wd, xd, n, path="mma"))
    np.testing.assert_array_equal(c2.view(np.uint32), c.view(np.uint32))
    if n % 32 == 0:
        q = host(pb.compute_out("q4_0", wd, xd, n, "q8_0", path="mma"))
        assert q.tobytes() == oracle.quantize("q8_0", c).tobytes()
    monkeypatch.setenv("PFNG_B200_GEMM_SPLITS", "1")
    c1 = host(pb.compute("q4_0", wd, xd, n, path="mma"))
    check_close(c1, oracle.mm("q4_0", w, a, m, n, k), oracle.bound("q4_0", w, a, m, n, k), f"unsplit {m}x{n}x{k}")


@pytest.mark.parametrize("layout", ["ggml", "planar", "q4_K"])
@pytest.mark.parametrize("m,n,k,splits", [(32, 1024, 4096, None), (32, 4000, 2048, "1"), (9, 300, 1536, "1"),
                                          (17, 640, 4096, None), (32, 130, 256, "1"), (40, 1000, 1536, None),
                                          (64, 2048, 4096, None), (130, 700, 2048, "1"), (480, 1536, 1536, None),
                                          (2048, 2048, 512, None), (1100, 3000, 1024, None)])
def test_direct_operands_equal_decode_pass(oracle, monkeypatch, layout, m, n, k, splits):
    # q4_0 and q4_K tiles (32, 64 and 128 rows) build the B fragments
    # straight from the raw W tile; PFNG_B200_GEMM_DIRECT=0 runs the decode
    # pass into the B tile (the two-phase or the overlapped kernel).  Same
    # products, same fold constants, same order: the same bits, and both
    # within tolerance of the oracle.
    if splits:
        monkeypatch.setenv("PFNG_B200_GEMM_SPLITS", splits)
    if layout == "q4_K" and k % 256 != 0:
        pytest.skip("q4_K needs k % 256 == 0")
    rng = np.random.default_rng(m * 5 + n + k)
    base = "q4_K" if layout == "q4_K" else "q4_0"
    w = oracle.quantize(base, rng.standard_normal((n, k)).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    a = oracle.quantize(act_kind(base), x)
    wd, xd = dev_bytes(w), dev(x)
    wt = base
    if layout == "planar":
        wd, wt = pb.pack_q4_0_planar(wd, n, k), "q4_0_planar"
    c = host(pb.compute(wt, wd, xd, n, path="mma"))
    check_close(c, oracle.mm(base, w, a, m, n, k), oracle.bound(base, w, a, m, n, k), f"direct {m}x{n}x{k}")
    monkeypatch.setenv("PFNG_B200_GEMM_DIRECT", "0")
    c0 = host(pb.compute(wt, wd, xd, n, path="mma"))
    np.testing.assert_array_equal(c.view(np.uint32), c0.view(np.uint32))
