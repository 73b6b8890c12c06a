"""GPU tier: tcgen05 GEMM parity with the oracle, through the C ABI (libmfb.so).

Mirrors the reference's GEMM tests (tests/unit/test_gemm_plan.cpp,
tests/unit/test_operations.cpp:30-47, tests/integration/test_infra.cpp:121-137) and adds
oracle parity on the golden fixtures and on seeded shapes (odd sizes, padded strides,
transposes, every epilogue, both precisions)."""
import ctypes
import threading

import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from helpers import STRICT_NORMWISE, assert_strict, assert_tf32, to_dev

pytestmark = pytest.mark.gpu

FP32, TF32 = mf.GemmPrecision.fp32, mf.GemmPrecision.tf32


def run_sgemm(m, n, k, a, lda, b, ldb, c0, ldc, alpha, beta, precision, ta=False, tb=False, epilogue=0, bias=None):
    """Runs mfb_sgemm on flat buffers laid out like the reference's pointer interface."""
    ar, ac = (k, m) if ta else (m, k)
    br, bc = (n, k) if tb else (k, n)

    def stored(buf, rows, ld):
        flat = np.zeros(max(rows, 1) * ld, np.float32)
        src = np.asarray(buf, np.float32).reshape(-1)[: flat.size]
        flat[: src.size] = src
        return to_dev(flat.reshape(max(rows, 1), ld))

    A = stored(a, ar, lda)[:ar, :ac]
    B = stored(b, br, ldb)[:br, :bc]
    Cfull = to_dev(np.asarray(c0, np.float32).reshape(m, ldc).copy())
    C = Cfull[:, :n]
    o = mf.GemmOptions(transpose_left=ta, transpose_right=tb, precision=precision, epilogue=mf.GemmEpilogue(epilogue))
    mf.sgemm(A, B, C, alpha, beta, o, to_dev(bias) if bias is not None else None)
    mf.sync()
    out = Cfull.cpu().numpy()
    assert np.array_equal(out[:, n:], np.asarray(c0, np.float32).reshape(m, ldc)[:, n:]), "row padding was written"
    return out[:, :n]


@pytest.mark.parametrize("precision", [FP32, TF32])
def test_golden_fixtures(golden_gemm, precision):
    for name, g in golden_gemm.items():
        m, n, k = int(g["m"]), int(g["n"]), int(g["k"])
        lda, ldb, ldc = int(g["lda"]), int(g["ldb"]), int(g["ldc"])
        alpha, beta = float(g["alpha"]), float(g["beta"])
        got = run_sgemm(m, n, k, g["a"], lda, g["b"], ldb, g["c_in"], ldc, alpha, beta, precision)
        ref32 = g["c_out"].reshape(m, ldc)[:, :n]
        if k == 0:
            assert np.array_equal(got, ref32), name
            continue
        a2 = g["a"][: m * lda].reshape(m, lda)[:, :k]
        b2 = g["b"][: k * ldb].reshape(k, ldb)[:, :n]
        if precision == FP32:
            ref64 = oracle.gemm_f64(m, n, k, g["a"], lda, g["b"], ldb, g["c_in"], ldc, alpha, beta)
            assert_strict(got, ref32, ref64, k, np.abs(a2).max(), np.abs(b2).max(), name)
        else:
            assert_tf32(got, ref32, name)


@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
@pytest.mark.parametrize("ep", [0, 1, 2, 3])
def test_plan_transpose_scaling_epilogues(golden_gemm, ta, tb, ep):
    """test_gemm_plan.cpp:14-34: 7x9x5, alpha 0.7, beta -0.3, C=ones, double dot at 3e-5."""
    g = golden_gemm["plan_7x9x5"]
    m, n, k = 7, 9, 5
    av, bv, biasv = g["a"], g["b"], g["bias"]
    a_store = av.reshape(m, k).T.copy() if ta else av.reshape(m, k)
    b_store = bv.reshape(k, n).T.copy() if tb else bv.reshape(k, n)
    a = to_dev(a_store)
    b = to_dev(b_store)
    bias = to_dev(biasv)
    c = torch.ones((m, n), device="cuda")
    o = mf.GemmOptions(transpose_left=ta, transpose_right=tb, epilogue=mf.GemmEpilogue(ep))
    plan = mf.GemmPlan(m, n, k, o)
    plan.execute(a, b, c, 0.7, -0.3, bias if ep else None)
    got = c.cpu().numpy()
    ref = 0.7 * (av.reshape(m, k).astype(np.float64) @ bv.reshape(k, n).astype(np.float64)) - 0.3
    if ep:
        ref = ref + biasv
    if ep == 2:
        ref = np.maximum(ref, 0.0)
    if ep == 3:
        ref = 0.5 * ref * (1 + np.tanh(0.7978845608 * (ref + 0.044715 * ref ** 3)))
    assert np.max(np.abs(got - ref)) <= 3e-5


def test_empty_inner_dimension_alias_and_validation():
    """test_gemm_plan.cpp:36-50."""
    a = torch.empty((3, 0), device="cuda")
    b = torch.empty((0, 4), device="cuda")
    c = torch.ones((3, 4), device="cuda")
    bias = torch.ones(4, device="cuda")
    empty = mf.GemmPlan(3, 4, 0, mf.GemmOptions(epilogue=mf.GemmEpilogue.bias_relu))
    empty.execute(a, b, c, 1, -2, bias)
    assert torch.all(c == 0)
    empty.execute(a, b, c, 1, 0, bias)
    assert torch.all(c == 1)
    square = torch.eye(3, device="cuda")
    p = mf.GemmPlan(3, 3, 3)
    with pytest.raises(mf.InvalidArgumentError):
        p.execute(square, square, square)
    with pytest.raises(mf.ShapeMismatchError):
        p.execute(square, b, c)
    with pytest.raises(mf.InvalidArgumentError):
        mf.GemmPlan(2 ** 31, 1, 1)
    moved = p.move()
    with pytest.raises(mf.InvalidArgumentError):
        p.execute(square, square, torch.zeros(3, 3, device="cuda"))
    out = torch.zeros(3, 3, device="cuda")
    moved.execute(square, square, out)
    torch.cuda.synchronize()
    assert torch.equal(out, square)
    with pytest.raises(mf.ShapeMismatchError):
        mf.GemmPlan(3, 3, 3, mf.GemmOptions(epilogue=mf.GemmEpilogue.bias)).execute(square, square, out)


def test_tune_preserves_output_and_graph_replay_reads_inputs():
    """test_gemm_plan.cpp:51-67."""
    torch.manual_seed(17)
    left = torch.rand(128, 128, device="cuda")
    right = torch.rand(128, 128, device="cuda")
    out = torch.ones(128, 128, device="cuda")
    plan = mf.GemmPlan(128, 128, 128, mf.GemmOptions(precision=TF32))
    tuning = plan.tune(left, right, out, 1, 0.5)
    assert tuning.candidates_tested > 0
    torch.cuda.synchronize()
    assert torch.all(out == 1)
    reference = mf.gemm(left, right)
    plan.execute(left, right, out)
    torch.cuda.synchronize()
    # A plan is bound to its stream: build one on the capture stream before capture.
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        cap_plan = mf.GemmPlan(128, 128, 128, mf.GemmOptions(precision=TF32))
        cap_plan.execute(left, right, out)
    s.synchronize()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=s):
        cap_plan.execute(left, right, out)
    g2.replay()
    torch.cuda.synchronize()
    assert torch.max(torch.abs(out - reference)).item() <= 0.025
    right.fill_(0)
    g2.replay()
    torch.cuda.synchronize()
    assert torch.all(out == 0)


@pytest.mark.parametrize("inner", [127, 2048])
def test_vector_times_matrix_strict(inner):
    """test_gemm_plan.cpp:68-80: 1 x inner x 127 at a strict double-dot tolerance of 2e-5."""
    rng = np.random.default_rng(91)
    v = (rng.random((1, inner)) - 0.5).astype(np.float32)
    w = (rng.random((inner, 127)) - 0.5).astype(np.float32)
    prod = mf.multiply(to_dev(v), to_dev(w)).cpu().numpy()
    ref = v.astype(np.float64) @ w.astype(np.float64)
    assert np.max(np.abs(prod - ref)) <= 2e-5


def test_concurrent_threads_isolated():
    """test_gemm_plan.cpp:81-88: two threads, 10 multiply_into each, results 512 and -768."""
    results = {}

    def worker(value):
        with torch.cuda.stream(torch.cuda.Stream()):
            x = torch.ones(256, 256, device="cuda") * value
            y = torch.ones(256, 256, device="cuda")
            z = torch.empty(256, 256, device="cuda")
            for _ in range(10):
                mf.multiply_into(x, y, z)
            torch.cuda.current_stream().synchronize()
            results[value] = z[127, 129].item()

    ts = [threading.Thread(target=worker, args=(v,)) for v in (2.0, -3.0)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert abs(results[2.0] - 512) < 0.01 and abs(results[-3.0] + 768) < 0.01


def test_operations_known_answers():
    """test_operations.cpp:30-47."""
    a = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda")
    b = torch.tensor([[2.0, 0.0], [1.0, 2.0]], device="cuda")
    out = torch.empty(2, 2, device="cuda")
    mf.multiply_into(a, b, out)
    assert out.cpu().tolist() == [[4.0, 4.0], [10.0, 8.0]]
    fused = mf.gemm_bias_relu(a, b, torch.tensor([[1.0, -10.0]], device="cuda"))
    assert fused.cpu().tolist() == [[5.0, 0.0], [11.0, 0.0]]


def test_infra_threads_ones_times_identity():
    """test_infra.cpp:121-137: 4 threads x 30 iterations of ones(24) * I(24), sum checked."""
    totals = [0.0] * 4

    def worker(i):
        with torch.cuda.stream(torch.cuda.Stream()):
            tot = 0.0
            for _ in range(30):
                c = mf.multiply(torch.ones(24, 24, device="cuda"), torch.eye(24, device="cuda"))
                tot += c.sum().item()
            totals[i] = tot

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert all(abs(t - 30 * 576) < 1e-2 for t in totals)


@pytest.mark.parametrize("precision", [FP32, TF32])
@pytest.mark.parametrize("m,n,k,pad", [(1, 300, 77, 0), (129, 17, 65, 3), (257, 383, 1000, 5), (640, 520, 333, 8),
                                       (1024, 1024, 4096, 32), (3, 1000, 2000, 1), (130, 250, 70, 0),
                                       (2100, 2200, 777, 4), (2304, 2048, 96, 0)])
def test_seeded_shapes_against_oracle(m, n, k, pad, precision):
    lda, ldb, ldc = k + pad, n + pad, n + 2 * pad
    a = oracle.seeded(m * lda, seed=m)
    b = oracle.seeded(k * ldb, "normal", seed=n)
    c0 = oracle.seeded(m * ldc, "normal", seed=k)
    got = run_sgemm(m, n, k, a, lda, b, ldb, c0, ldc, 0.5, 1.0, precision)
    ref32 = c0.copy()
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, ref32, ldc, 0.5, 1.0,
                    impl="reference" if oracle.reference_available() else "restatement")
    ref32 = ref32.reshape(m, ldc)[:, :n]
    if precision == FP32:
        ref64 = oracle.gemm_f64(m, n, k, a, lda, b, ldb, c0, ldc, 0.5, 1.0)
        assert_strict(got, ref32, ref64, k, np.abs(a).max(), np.abs(b).max(), f"{m}x{n}x{k}")
    else:
        assert_tf32(got, ref32, f"{m}x{n}x{k}")


@pytest.mark.parametrize("ta,tb", [(True, False), (False, True), (True, True)])
def test_transposed_operands_against_oracle(ta, tb):
    m, n, k = 300, 260, 513
    a = oracle.seeded((m, k), seed=1)
    b = oracle.seeded((k, n), seed=2)
    a_store = a.T.copy() if ta else a
    b_store = b.T.copy() if tb else b
    got = run_sgemm(m, n, k, a_store, a_store.shape[1], b_store, b_store.shape[1], np.zeros((m, n), np.float32), n,
                    1.0, 0.0, FP32, ta, tb)
    ref32 = np.zeros(m * n, np.float32)
    oracle.gemm_f32(m, n, k, a, k, b, n, ref32, n)
    assert_strict(got, ref32.reshape(m, n), oracle.gemm_f64(m, n, k, a, k, b, n), k, 1.0, 1.0)


def test_cuda_gemm_drop_in_with_padded_strides():
    """matrix_pro::hw::cuda_gemm semantics: device pointers, padded lda/ldb/ldc, async + cuda_sync."""
    m, n, k, lda, ldb, ldc = 200, 300, 400, 432, 320, 310
    a = oracle.seeded(m * lda, seed=3)
    b = oracle.seeded(k * ldb, "normal", seed=4)
    c0 = oracle.seeded(m * ldc, "normal", seed=5)
    A, B, C = to_dev(a), to_dev(b), to_dev(c0.copy())
    mf.cuda_gemm(0, m, n, k, A.data_ptr(), lda, B.data_ptr(), ldb, C.data_ptr(), ldc, 0.5, 1.0)
    mf.cuda_sync(0)
    got = C.cpu().numpy().reshape(m, ldc)
    ref = c0.copy()
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, ref, ldc, 0.5, 1.0)
    ref = ref.reshape(m, ldc)
    assert np.array_equal(got[:, n:], ref[:, n:])
    assert_strict(got[:, :n], ref[:, :n], oracle.gemm_f64(m, n, k, a, lda, b, ldb, c0, ldc, 0.5, 1.0), k,
                  np.abs(a).max(), np.abs(b).max())
    with pytest.raises(mf.InvalidArgumentError):
        mf.cuda_gemm(99, m, n, k, A.data_ptr(), lda, B.data_ptr(), ldb, C.data_ptr(), ldc, 1.0, 0.0)


def test_naive_device_oracle_matches_restatement_bit_exact():
    """alpha 1, beta 0, n a multiple of 16: both are one FP32 FMA chain over k per output."""
    m, n, k = 96, 64, 777
    a = oracle.seeded((m, k), seed=7)
    b = oracle.seeded((k, n), seed=8)
    out = torch.empty(m, n, device="cuda")
    mf.naive_sgemm(to_dev(a), to_dev(b), out)
    ref = np.zeros(m * n, np.float32)
    oracle.gemm_f32(m, n, k, a, k, b, n, ref, n)
    assert np.array_equal(out.cpu().numpy(), ref.reshape(m, n))


def test_plan_info_and_no_tcgen05_for_vectors():
    p = mf.GemmPlan(512, 512, 512)
    info = p.info()
    assert info.kernel.decode() == "tcgen05_3xtf32" and info.tile_n in (64, 128, 256) and p.uses_tcgen05()
    assert info.workspace_bytes >= 2 * 2 * 512 * 512 * 4  # hi and lo planes of A and B
    big = mf.GemmPlan(8192, 11008, 4096)
    assert big.info().tile_n == 256 and big.candidate_count() >= 2  # SM-pair and single-CTA tilings
    v = mf.GemmPlan(512, 1, 512)
    assert v.info().kernel.decode() == "gemv_fp32" and not v.uses_tcgen05()
    t = mf.GemmPlan(4096, 4096, 64, mf.GemmOptions(precision=TF32))
    assert t.info().kernel.decode() == "tcgen05_tf32"
    assert t.info().workspace_bytes >= (4096 * 64 + 64 * 4096) * 4  # one rounded TF32 plane per operand


@pytest.mark.parametrize("precision", [FP32, TF32])
def test_prepare_operands_one_at_a_time(precision):
    """mfb_plan_prepare with a NULL operand prepares only the other one (A before B, as the
    row split does while B is still arriving); the multiply then equals mfb_plan_execute."""
    from matrixflash_pro_b200 import _lib
    from matrixflash_pro_b200.gemm import _stream_handle
    m, n, k = 300, 520, 700
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn((m, k), device="cuda", generator=g)
    B = torch.randn((k, n), device="cuda", generator=g)
    C0 = torch.randn((m, n), device="cuda", generator=g)
    p = mf.GemmPlan(m, n, k, mf.GemmOptions(precision=precision))
    # Column ranges run whole tiles; compare with the plan's first candidate that does too
    # (a stream-K launch adds the K shares in another order).
    for i in range(p.candidate_count()):
        p.select_candidate(i)
        if p.info().stream_k_tiles == 0:
            break
    assert p.info().stream_k_tiles == 0
    want = C0.clone()
    p.execute(A, B, want, 0.5, 1.0)
    got = C0.clone()
    lib, h, s = _lib.lib(), p._handle, _stream_handle()
    _lib.check(lib.mfb_plan_prepare(h, s, A.data_ptr(), 0), "prepare A")
    _lib.check(lib.mfb_plan_prepare(h, s, 0, B.data_ptr()), "prepare B")
    _lib.check(lib.mfb_plan_multiply(h, s, A.data_ptr(), B.data_ptr(), got.data_ptr(), 0.5, 1.0, 0), "multiply")
    mf.sync()
    assert torch.equal(got, want)
    with pytest.raises(mf.InvalidArgumentError):
        _lib.check(lib.mfb_plan_prepare(h, s, 0, 0), "prepare nothing")


def test_tf32_mma_rate_probe():
    """The diagnostic TF32 MMA-rate probe returns a plausible B200 figure and leaves no status bit."""
    peak256 = mf.probe_tf32_mma_tflops(256)
    peak64 = mf.probe_tf32_mma_tflops(64)
    assert 300.0 < peak256 < 1500.0, peak256
    assert 0.0 < peak64 < peak256  # narrow MMAs cost nearly as long as wide ones
    assert mf.device_status() == 0
    with pytest.raises(mf.InvalidArgumentError):
        mf.probe_tf32_mma_tflops(96)


@pytest.mark.parametrize("precision", [FP32, TF32])
def test_column_range_phases_equal_execute(precision):
    """mfb_plan_prepare_cols / mfb_plan_multiply_cols (B arriving in contiguous column panels,
    as the row split broadcasts it) give the bits of one mfb_plan_execute."""
    from matrixflash_pro_b200 import _lib
    from matrixflash_pro_b200.gemm import _stream_handle
    m, n, k = 1000, 2000, 700
    g = torch.Generator(device="cuda").manual_seed(12)
    A = torch.randn((m, k), device="cuda", generator=g)
    B = torch.randn((k, n), device="cuda", generator=g)
    C0 = torch.randn((m, n), device="cuda", generator=g)
    p = mf.GemmPlan(m, n, k, mf.GemmOptions(precision=precision))
    # Column ranges run whole tiles; compare with the plan's first candidate that does too
    # (a stream-K launch adds the K shares in another order).
    for i in range(p.candidate_count()):
        p.select_candidate(i)
        if p.info().stream_k_tiles == 0:
            break
    assert p.info().stream_k_tiles == 0
    want = C0.clone()
    p.execute(A, B, want, 0.5, 1.0)
    lib, h, s = _lib.lib(), p._handle, _stream_handle()
    got = C0.clone()
    _lib.check(lib.mfb_plan_prepare(h, s, A.data_ptr(), 0), "prepare A")
    for n0, n1 in [(512, 2000), (0, 512)]:
        Bp = B[:, n0:n1].contiguous()
        _lib.check(lib.mfb_plan_prepare_cols(h, s, Bp.data_ptr(), n1 - n0, n0, n1), "prepare cols")
        _lib.check(lib.mfb_plan_multiply_cols(h, s, A.data_ptr(), got.data_ptr(), 0.5, 1.0, 0, n0, n1),
                   "multiply cols")
        mf.sync()  # Bp is freed at the end of the iteration
    assert torch.equal(got, want)
    with pytest.raises(mf.InvalidArgumentError):
        _lib.check(lib.mfb_plan_multiply_cols(h, s, A.data_ptr(), got.data_ptr(), 1.0, 0.0, 0, 16, 64), "n0")
    with pytest.raises(mf.InvalidArgumentError):
        _lib.check(lib.mfb_plan_prepare_cols(h, s, B.data_ptr(), n, 0, n + 32), "n1")


@pytest.mark.parametrize("precision", [FP32, TF32])
@pytest.mark.parametrize("ta,tb", [(True, True), (False, False), (True, False)])
def test_sm_pair_transposed_operands(ta, tb, precision):
    """256 x 256 SM-pair tiles with MN-major A and/or K-major B (2048 x 2048 outputs fill the pairs)."""
    m, n, k = 2048, 2048, 544
    g = torch.Generator(device="cuda").manual_seed(31 + 2 * ta + tb)
    A = torch.randn((k, m) if ta else (m, k), device="cuda", generator=g)
    B = torch.randn((n, k) if tb else (k, n), device="cuda", generator=g)
    C0 = torch.randn((m, n), device="cuda", generator=g)
    o = mf.GemmOptions(precision=precision, transpose_left=ta, transpose_right=tb)
    p = mf.GemmPlan(m, n, k, o)
    assert p.info().sm_pair == 1
    C = C0.clone()
    p.execute(A, B, C, 0.75, -0.5)
    mf.sync()
    Ad = A.double().t() if ta else A.double()
    Bd = B.double().t() if tb else B.double()
    ref = 0.75 * (Ad @ Bd) - 0.5 * C0.double()
    err = float((C.double() - ref).norm() / ref.norm())
    assert err <= (STRICT_NORMWISE if precision == FP32 else 5e-3), err
