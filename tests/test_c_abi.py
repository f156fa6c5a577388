"""Host-side behaviour of the C ABI (include/pfng_b200.h), no GPU needed.

The library must load, export every function the header declares, and reject
bad arguments on the host -- before any CUDA call -- with the documented
status codes.  These mirror the reference's fail-closed conventions
(validate -> SKIP with a reason, prepare -> error string;
bench/framework/kernel_registry.h:71-84).
"""
import ctypes

import pytest

import pfng_b200 as pb

OK, INVALID, SHAPE, ALIGN, WORKSPACE = 0, -1, -2, -3, -4


@pytest.fixture(scope="module")
def L():
    return pb.lib()


def test_library_exports_every_header_symbol(L):
    names = pb.header_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(L, name), f"{name} declared in include/pfng_b200.h but not exported"


def test_version_and_status_strings(L):
    assert L.pfng_b200_version() >= 1
    assert pb.status_string(0) == "ok"
    assert "shape" in pb.status_string(SHAPE)
    assert "aligned" in pb.status_string(ALIGN)
    assert "workspace" in pb.status_string(WORKSPACE)


FAKE = 0x10000  # never dereferenced: every call below is rejected on the host


@pytest.mark.parametrize("fn,k", [("pfng_b200_mm_q4_0_q8_0", 33), ("pfng_b200_mm_q4_K_q8_K", 32),
                                  ("pfng_b200_mm_iq2_xxs_q8_K", 128)])
def test_mm_rejects_k_not_multiple_of_block(L, fn, k):
    assert getattr(L, fn)(FAKE, FAKE, FAKE, 4, 4, k, 4, None, 0, 0, None) == SHAPE


def test_mm_argument_checks(L):
    f = L.pfng_b200_mm_q4_0_q8_0
    assert f(FAKE, FAKE, FAKE, -1, 4, 32, 4, None, 0, 0, None) == INVALID
    assert f(FAKE, FAKE, FAKE, 4, 4, 32, 3, None, 0, 0, None) == SHAPE          # ldc < n
    assert f(None, FAKE, FAKE, 4, 4, 32, 4, None, 0, 0, None) == INVALID        # null W
    assert f(FAKE, FAKE, FAKE + 2, 4, 4, 32, 4, None, 0, 0, None) == ALIGN      # C not 4-aligned
    assert f(FAKE + 1, FAKE, FAKE, 4, 4, 32, 4, None, 0, 0, None) == ALIGN      # W not 2-aligned
    assert f(FAKE, FAKE, FAKE, 4, 4, 32, 4, None, 0, 9, None) == INVALID        # unknown path
    # empty problems are valid no-ops and touch nothing
    assert f(None, None, None, 0, 4, 32, 4, None, 0, 0, None) == OK
    assert f(None, None, None, 4, 0, 32, 4, None, 0, 0, None) == OK
    g = L.pfng_b200_mm_q4_K_q8_K
    assert g(FAKE + 2, FAKE, FAKE, 4, 4, 256, 4, None, 0, 0, None) == ALIGN     # q4_K blocks are 4-aligned
    h = L.pfng_b200_mm_iq2_xxs_q8_K
    assert h(FAKE, FAKE + 2, FAKE, 4, 4, 256, 4, None, 0, 0, None) == ALIGN     # q8_K blocks are 4-aligned


def test_compute_argument_checks(L):
    f = L.pfng_b200_compute_q4_0
    assert f(FAKE, FAKE, 16, FAKE, 4, 4, 32, 4, None, 0, 0, None) == SHAPE      # ldx < k
    assert f(FAKE, FAKE + 2, 32, FAKE, 4, 4, 32, 4, None, 0, 0, None) == ALIGN  # fp32 x misaligned


def test_quantizer_argument_checks(L):
    assert L.pfng_b200_quantize_q8_0(FAKE, 48, FAKE, 2, 48, None) == SHAPE
    assert L.pfng_b200_quantize_q8_K(FAKE, 512, FAKE, 2, 384, None) == SHAPE
    assert L.pfng_b200_quantize_q8_K(FAKE, 256, FAKE + 2, 2, 256, None) == ALIGN
    assert L.pfng_b200_quantize_q4_0(FAKE, 16, FAKE, 2, 32, None) == SHAPE      # ldx < k
    assert L.pfng_b200_quantize_q4_K(None, 256, FAKE, 2, 256, None) == INVALID
    assert L.pfng_b200_quantize_q8_0(None, 32, None, 0, 32, None) == OK


def test_valid_call_without_gpu_reports_cuda_error(L):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st = L.pfng_b200_quantize_q8_0(FAKE, 32, FAKE, 1, 32, None)
    assert st <= -1000, st  # a CUDA error surfaced as a status, no crash


def test_workspace_sizes(L):
    assert pb.mm_workspace_size("q4_0", 1, 4096, 4096) == 0            # GEMV needs none
    big = pb.mm_workspace_size("q4_0", 480, 1536, 1536)
    assert big >= 512 * 1536                                            # split int8 rows, padded to 128
    assert pb.compute_workspace_size("q4_K", 1, 4096, 4096) > 0         # simple-path fallback room
    assert pb.mm_workspace_size("q4_0", 0, 4, 32) == 0


@pytest.mark.parametrize("n,world,granule", [(4096, 8, 128), (11008, 3, 128), (100, 8, 32), (5, 4, 1), (0, 2, 8)])
def test_shard_rows_partition(n, world, granule):
    spans = [pb.shard_rows(n, world, r, granule) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
        assert e0 == b1 and b0 <= e0
    for b, _ in spans:
        assert b % granule == 0 or b == n
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= granule


def test_shard_rows_rejects_bad_rank():
    with pytest.raises(pb.PfngError):
        pb.shard_rows(10, 2, 2, 1)


def test_planar_argument_checks(L):
    pack, unpack = L.pfng_b200_pack_q4_0_planar, L.pfng_b200_unpack_q4_0_planar
    big = FAKE * 16
    assert pack(FAKE, big, 4, 96, None) == SHAPE            # k % 256 != 0
    assert pack(FAKE, big + 2, 4, 256, None) == ALIGN       # planar side 16-byte aligned
    assert pack(FAKE + 1, big, 4, 256, None) == ALIGN       # ggml side 2-byte aligned
    assert unpack(big + 8, FAKE, 4, 256, None) == ALIGN
    assert pack(FAKE, FAKE + 16, 4, 256, None) == INVALID   # overlapping buffers
    assert pack(None, big, 4, 256, None) == INVALID
    assert pack(None, None, 0, 256, None) == OK
    assert pack(FAKE, big, -1, 256, None) == INVALID
    mm = L.pfng_b200_mm_q4_0p_q8_0
    assert mm(FAKE, FAKE, FAKE, 4, 4, 32, 4, None, 0, 0, None) == SHAPE      # planar needs k % 256 == 0
    assert mm(FAKE + 2, FAKE, FAKE, 4, 4, 256, 4, None, 0, 0, None) == ALIGN  # planar W 16-byte aligned
    assert mm(FAKE, FAKE + 1, FAKE, 4, 4, 256, 4, None, 0, 0, None) == ALIGN  # q8_0 blocks 2-aligned
    comp = L.pfng_b200_compute_q4_0p
    assert comp(FAKE, FAKE, 128, FAKE, 4, 4, 256, 4, None, 0, 0, None) == SHAPE  # ldx < k
    part = L.pfng_b200_partials_q4_0p_q8_0
    assert part(None, None, None, 0, 4, 256, None, 0, 0, None) == OK
    # weight type code 3 is the planar layout, 4 is unknown
    assert pb.mm_workspace_size("q4_0_planar", 480, 1536, 1536) == pb.mm_workspace_size("q4_0", 480, 1536, 1536)
    assert pb.mm_workspace_size(4, 480, 1536, 1536) == 0
    grouped = L.pfng_b200_compute_grouped
    n = (ctypes.c_int64 * 1)(4)
    ptrs = (ctypes.c_void_p * 1)(FAKE)
    ldc = (ctypes.c_int64 * 1)(4)
    assert grouped(4, 1, ptrs, n, ptrs, ldc, FAKE, 256, 1, 256, 0, None) == INVALID
    assert grouped(3, 1, ptrs, n, ptrs, ldc, FAKE, 256, 1, 96, 0, None) == SHAPE


def test_output_format_argument_checks(L):
    mm, comp = L.pfng_b200_mm_out, L.pfng_b200_compute_out
    assert mm(0, FAKE, FAKE, FAKE, 4, 64, 4, 64, 256, None, 0, 0, None) == INVALID      # unknown format
    assert mm(0, FAKE, FAKE, FAKE, 3, 2, 4, 48, 256, None, 0, 0, None) == SHAPE        # q8_0 needs n % 32 == 0
    assert mm(0, FAKE, FAKE, FAKE, 3, 1, 4, 64, 256, None, 0, 0, None) == SHAPE        # ldo < n / 32 blocks
    assert mm(0, FAKE, FAKE, FAKE, 1, 63, 4, 64, 256, None, 0, 0, None) == SHAPE       # ldo < n halves
    assert mm(0, FAKE, FAKE, FAKE + 1, 1, 64, 4, 64, 256, None, 0, 0, None) == ALIGN   # 2-byte outputs
    assert mm(0, FAKE + 1, FAKE, FAKE, 1, 64, 4, 64, 256, None, 0, 0, None) == ALIGN   # W still checked
    assert mm(0, None, FAKE, FAKE, 2, 64, 4, 64, 256, None, 0, 0, None) == INVALID
    assert mm(0, None, None, None, 3, 2, 0, 64, 256, None, 0, 0, None) == OK          # empty
    assert comp(0, FAKE, FAKE, 128, FAKE, 1, 64, 4, 64, 256, None, 0, 0, None) == SHAPE  # ldx < k
    # workspace: GEMV / SIMPLE keep an fp32 C scratch, the tensor-core GEMM converts in its epilogue
    assert pb.lib().pfng_b200_compute_out_workspace_size(0, 1, 1, 4096, 4096, 1) >= 4096 * 4
    assert pb.lib().pfng_b200_compute_out_workspace_size(0, 0, 1, 4096, 4096, 1) == 0
    fused = pb.lib().pfng_b200_compute_out_workspace_size(0, 3, 480, 1536, 1536, 2)
    assert fused == pb.compute_workspace_size("q4_0", 480, 1536, 1536, "mma")


def test_selftest_wait_rejects_zero_attempts(L):
    # checked on the host before any CUDA call
    assert L.pfng_b200_selftest_wait(0, 1, None, None) == INVALID
