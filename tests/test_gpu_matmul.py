"""GPU parity of float32 matmul against the CPU oracle, both kernels.

Bar: relative Frobenius error <= 1e-4 * sqrt(K / 1024) (at least the 1e-4 floor)
against the CPU reference, plus the reference tests' elementwise check
(rtol = atol = 1e-4, tests/python/test_cuda_primitives.py:9-21 and
test_batched_matmul.py:14-50)."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PATHS = ["ffma", "tensor"]


def dev(a):
    return torch.from_numpy(np.array(a, order="C")).cuda()  # keeps 0-d arrays 0-d


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def frob_ok(got, ref, k):
    tol = 1e-4 * math.sqrt(max(k, 1024) / 1024)
    num = np.linalg.norm((got.astype(np.float64) - ref.astype(np.float64)).ravel())
    den = np.linalg.norm(ref.astype(np.float64).ravel())
    assert num <= tol * max(den, 1e-30), (num / max(den, 1e-30), tol)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (2, 3, 4), (15, 17, 31), (17, 16, 15), (32, 33, 16), (0, 3, 4),
                                   (3, 0, 4), (3, 4, 0), (65, 129, 67)])
def test_reference_shapes(tcx, oracle, path, m, k, n):
    rng = np.random.default_rng(7)
    a = rng.normal(size=(m, k)).astype(np.float32)
    b = rng.normal(size=(k, n)).astype(np.float32)
    got = host(tcx.matmul(dev(a), dev(b), path=path))
    assert got.shape == (m, n)
    np.testing.assert_allclose(got, oracle.matmul(a, b), rtol=1e-4, atol=1e-4)


CASES = [((3,), (3,)), ((2, 3), (3,)), ((3,), (3, 4)), ((2, 3, 4), (2, 4, 5)), ((2, 3, 4), (4, 5)),
         ((3, 4), (2, 4, 5)), ((4,), (2, 4, 5)), ((2, 3, 4), (4,)), ((2, 1, 3, 4), (1, 5, 4, 6)),
         ((1, 2, 3, 4), (3, 1, 4, 5)), ((2, 1, 1, 3, 4), (1, 5, 1, 4, 2)), ((2, 17, 19), (1, 19, 33)),
         ((2, 33, 17), (2, 17, 1)), ((0,), (0,)), ((2, 0), (0,)), ((0,), (0, 3)), ((2, 3, 0), (1, 0, 4)),
         ((0, 3, 4), (1, 4, 2)), ((1, 3, 4), (0, 4, 2)), ((2, 0, 4), (2, 4, 3)), ((2, 3, 4), (2, 4, 0)),
         ((0, 2, 3, 0), (1, 2, 0, 4)), ((2, 1, 0, 3), (1, 5, 3, 4)), ((3,), (0, 3, 4)), ((0, 2, 3), (3,)),
         ((2, 1, 3, 4), (5, 4, 2))]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("shapes", CASES)
def test_batched_broadcast(tcx, oracle, path, shapes):
    rng = np.random.default_rng(741)
    a, b = [rng.uniform(-1, 1, s).astype(np.float32) for s in shapes]
    got = host(tcx.matmul(dev(a), dev(b), path=path))
    expected = oracle.matmul(a, b)
    assert got.shape == expected.shape
    np.testing.assert_allclose(got, expected, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("path", PATHS)
def test_special_values(tcx, oracle, path):
    a = np.array([[[np.nan, 1]], [[np.inf, 1]], [[-np.inf, -1]], [[-0., 0.]]], np.float32)
    b = np.array([[1.], [2.]], np.float32)
    got = host(tcx.matmul(dev(a), dev(b), path=path))
    np.testing.assert_allclose(got, oracle.matmul(a, b), rtol=1e-4, atol=1e-4, equal_nan=True)


@pytest.mark.parametrize("path", PATHS)
def test_inf_in_large_product_takes_ieee_path(tcx, oracle, path):
    rng = np.random.default_rng(2)
    a = rng.uniform(-1, 1, (256, 512)).astype(np.float32)
    b = rng.uniform(-1, 1, (512, 256)).astype(np.float32)
    a[3, 7] = np.inf
    got = host(tcx.matmul(dev(a), dev(b), path=path))
    expected = oracle.matmul(a, b)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(expected))
    np.testing.assert_array_equal(np.isinf(got), np.isinf(expected))
    fin = np.isfinite(expected)
    np.testing.assert_allclose(got[fin], expected[fin], rtol=1e-4, atol=1e-4)


def test_high_rank_and_grid_stride(tcx):
    a = torch.ones((1,) * 60 + (2, 3), device="cuda")  # torch caps tensors at 64 dims
    b = torch.ones((3, 4), device="cuda")
    r = tcx.matmul(a, b)
    assert tuple(r.shape) == (1,) * 60 + (2, 4)
    np.testing.assert_array_equal(host(r).reshape(2, 4), np.full((2, 4), 3, np.float32))
    values = (np.arange(65537, dtype=np.float32) % 17).reshape(-1, 1, 1)
    r = tcx.matmul(dev(values), dev(np.array([[2.]], np.float32)))
    np.testing.assert_array_equal(host(r), values * 2)
    with pytest.raises(ValueError):
        tcx.matmul(torch.empty((2, 3), device="cuda"), torch.empty((2, 3), device="cuda"))


@pytest.mark.parametrize("m,n,k", [(128, 256, 32), (256, 512, 128), (300, 300, 300), (129, 257, 33),
                                   (512, 512, 1024), (1024, 1024, 1024), (2048, 2048, 2048), (1000, 4000, 100),
                                   (384, 1280, 4096)])
def test_tensor_path_sizes(tcx, oracle, m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    got = host(tcx.matmul(dev(a), dev(b), path="tensor"))
    rows = slice(0, m) if m * n * k <= (1 << 28) else slice(m // 2 - 64, m // 2 + 64)
    ref = oracle.matmul(a, b, rows=rows, batches=[0])[0]
    frob_ok(got[rows], ref, k)
    np.testing.assert_allclose(got[rows], ref, rtol=2e-4 * math.sqrt(k / 1024) + 1e-4, atol=1e-4 * math.sqrt(k))


def test_tensor_path_is_more_accurate_than_tf32(tcx, oracle):
    """3xTF32 must land far below single-pass TF32 error (~3e-4 here). The tensor
    core adds each MMA into the float32 accumulator with truncation, so the error
    grows with K/8 accumulation steps (~1.5e-5 at K = 2048), still an order of
    magnitude inside the 1e-4 * sqrt(K/1024) bar."""
    rng = np.random.default_rng(4)
    a = rng.uniform(-1, 1, (256, 2048)).astype(np.float32)
    b = rng.uniform(-1, 1, (2048, 256)).astype(np.float32)
    got = host(tcx.matmul(dev(a), dev(b), path="tensor")).astype(np.float64)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    rel = np.linalg.norm(got - exact) / np.linalg.norm(exact)
    assert rel < 4e-5, rel


def test_batched_tensor_and_epilogue(tcx, oracle):
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (4, 256, 384)).astype(np.float32)
    b = rng.uniform(-1, 1, (4, 384, 512)).astype(np.float32)
    bias = rng.normal(size=512).astype(np.float32)
    for path in PATHS:
        for act in ("none", "silu", "relu"):
            got = host(tcx.matmul(dev(a), dev(b), bias=dev(bias), act=act, path=path))
            ref = oracle.add(oracle.matmul(a, b), bias)
            if act == "silu":
                ref = oracle.silu(ref)
            elif act == "relu":
                ref = oracle.relu(ref)
            frob_ok(got, ref, 384)


def test_broadcast_rhs_tensor_path(tcx, oracle):
    rng = np.random.default_rng(6)
    a = rng.uniform(-1, 1, (3, 200, 160)).astype(np.float32)
    b = rng.uniform(-1, 1, (160, 300)).astype(np.float32)
    frob_ok(host(tcx.matmul(dev(a), dev(b), path="tensor")), oracle.matmul(a, b), 160)
    a2 = rng.uniform(-1, 1, (2, 1, 130, 64)).astype(np.float32)
    b2 = rng.uniform(-1, 1, (1, 3, 64, 140)).astype(np.float32)
    frob_ok(host(tcx.matmul(dev(a2), dev(b2), path="tensor")), oracle.matmul(a2, b2), 64)


@pytest.mark.parametrize("path", ["auto", "ffma", "tensor"])
@pytest.mark.parametrize("shape", [(256, 784, 512), (256, 512, 10), (3, 7, 5), (2, 130, 300, 200)])
def test_linear_fused(tcx, oracle, path, shape):
    """linear reads the [out, in] weight in place (no transpose copy) with the bias in
    the GEMM epilogue; equals the reference composite transpose -> matmul -> add."""
    rng = np.random.default_rng(8)
    *lead, fin, fout = shape
    x = rng.normal(size=(*lead, fin)).astype(np.float32)
    w = rng.uniform(-1 / np.sqrt(fin), 1 / np.sqrt(fin), (fout, fin)).astype(np.float32)
    b = rng.normal(size=fout).astype(np.float32)
    got = host(tcx.linear(dev(x), dev(w), dev(b), path=path))
    assert got.shape == (*lead, fout)
    frob_ok(got, oracle.linear(x, w, b), fin)


@pytest.mark.parametrize("m,n,k", [(4096, 1024, 512), (1000, 300, 70), (5, 7, 3), (2048, 2048, 0),
                                   (2048, 5000, 512), (512, 9728, 256)])
def test_matmul_host_pipeline(tcx, oracle, m, n, k):
    """Host-buffer matmul (chunked upload / GEMM / download pipeline) against the CPU
    oracle on sampled rows and against the device-buffer path (the same 3xTF32 products;
    the chunks' tiles split k differently from the whole product's when stream-K
    applies, so the two agree within the tolerance, not bit for bit); repeatable bit
    for bit. (2048, 5000, 512): 256-row chunks through the single-SM kernel's TMA-store
    epilogue; (512, 9728, 256): one chunk, a CTA-pair product."""
    rng = np.random.default_rng(m + n)
    a = torch.from_numpy(rng.uniform(-1, 1, (m, k)).astype(np.float32)).pin_memory()
    b = torch.from_numpy(rng.uniform(-1, 1, (k, n)).astype(np.float32)).pin_memory()
    c = tcx.matmul_host(a, b).numpy()
    rows = slice(0, m) if m <= 1024 else slice(m - 300, m)
    ref = oracle.matmul(a.numpy(), b.numpy(), rows=rows, batches=[0])[0]
    if k == 0:
        np.testing.assert_array_equal(c[rows], ref)
    else:
        frob_ok(c[rows], ref, k)
    dev = host(tcx.matmul(a.cuda(), b.cuda()))
    if k == 0:
        np.testing.assert_array_equal(c, dev)
    else:
        frob_ok(c, dev, k)
    np.testing.assert_array_equal(tcx.matmul_host(a, b).numpy(), c)


@pytest.mark.parametrize("lhs,rhs", [((2050, 130), (130, 2100)), ((1280, 1100), (1100, 2000)),
                                     ((3, 700, 900), (900, 1100)), ((2, 1, 600, 96), (1, 3, 96, 1000))])
def test_cta_pair_tiles_ragged_and_batched(tcx, oracle, lhs, rhs):
    """Products large enough for the CTA-pair kernel (256 x 256 tiles on two SMs), with
    ragged M and N edges and broadcast batches."""
    rng = np.random.default_rng(lhs[-1] + rhs[-1])
    a = rng.uniform(-1, 1, lhs).astype(np.float32)
    b = rng.uniform(-1, 1, rhs).astype(np.float32)
    got = host(tcx.matmul(dev(a), dev(b), path="tensor"))
    m = lhs[-2]
    if a.ndim == 2:
        ref = oracle.matmul(a, b, rows=slice(m - 300, m), batches=[0])[0]
        frob_ok(got[m - 300:], ref, lhs[-1])
    else:
        frob_ok(got, oracle.matmul(a, b), lhs[-1])


@pytest.mark.parametrize("lhs,rhs,act", [((4096, 1024), (1024, 4096), "relu"), ((2050, 1000), (1000, 2100), "silu"),
                                         ((3, 1024, 1024), (3, 1024, 2048), "silu"), ((1280, 1100), (1100, 2000), "none")])
def test_stream_k_tiles(tcx, oracle, lhs, rhs, act):
    """CTA-pair products whose last wave of 256 x 256 tiles leaves at least half of the
    clusters idle (256, 81 and 96 tiles over 74 clusters): the k-blocks of that wave and
    one whole wave before it are spread evenly over every cluster (stream-K); a tile
    split over two clusters is finished by the one holding its last k-block, which adds
    the other's partial accumulator before bias / activation. 40 tiles: no stream-K. Rows
    of whole-wave and stream-K tiles (ragged edges included) against the oracle; a second
    call is bit identical (the partial counters are reset per call)."""
    rng = np.random.default_rng(lhs[-1] + rhs[-1])
    a = rng.uniform(-1, 1, lhs).astype(np.float32)
    b = rng.uniform(-1, 1, rhs).astype(np.float32)
    n, k, m = rhs[-1], lhs[-1], lhs[-2]
    bias = rng.normal(size=n).astype(np.float32)
    ad, bd, biasd = dev(a), dev(b), dev(bias)
    got = host(tcx.matmul(ad, bd, bias=biasd, act=act, path="tensor"))
    post = {"none": lambda x: x, "relu": oracle.relu, "silu": oracle.silu}[act]
    if a.ndim == 2:
        for rows in (slice(0, 256), slice(m - 300, m)):
            ref = post(oracle.add(oracle.matmul(a, b, rows=rows, batches=[0])[0], bias))
            frob_ok(got[rows], ref, k)
    else:
        frob_ok(got, post(oracle.add(oracle.matmul(a, b), bias)), k)
    np.testing.assert_array_equal(host(tcx.matmul(ad, bd, bias=biasd, act=act, path="tensor")), got)


def test_stream_k_shape_with_nan_takes_ieee_path(tcx, oracle):
    """A NaN in an operand of a stream-K-eligible product: the pre-pass raises the flag,
    the pair kernel does no work (no partials, no counters) and the IEEE kernel behind
    it computes the product; rows of both wave kinds against the oracle. The next call,
    with the NaN replaced, runs stream-K again (its flag and counters reset per call)."""
    rng = np.random.default_rng(21)
    a = rng.uniform(-1, 1, (4096, 1024)).astype(np.float32)
    b = rng.uniform(-1, 1, (1024, 4096)).astype(np.float32)
    a[4000, 5] = np.nan
    got = host(tcx.matmul(dev(a), dev(b)))
    for rows in (slice(0, 64), slice(3990, 4010)):
        expected = oracle.matmul(a, b, rows=rows, batches=[0])[0]
        np.testing.assert_array_equal(np.isnan(got[rows]), np.isnan(expected))
        fin = np.isfinite(expected)
        np.testing.assert_allclose(got[rows][fin], expected[fin], rtol=1e-4, atol=1e-4)
    a[4000, 5] = 0.5
    got = host(tcx.matmul(dev(a), dev(b)))
    rows = slice(4096 - 300, 4096)
    frob_ok(got[rows], oracle.matmul(a, b, rows=rows, batches=[0])[0], 1024)


def test_cta_pair_epilogue_and_linear(tcx, oracle):
    rng = np.random.default_rng(12)
    a = rng.uniform(-1, 1, (4, 520, 384)).astype(np.float32)
    b = rng.uniform(-1, 1, (4, 384, 1030)).astype(np.float32)
    bias = rng.normal(size=1030).astype(np.float32)
    got = host(tcx.matmul(dev(a), dev(b), bias=dev(bias), act="relu", path="tensor"))
    frob_ok(got, oracle.relu(oracle.add(oracle.matmul(a, b), bias)), 384)
    x = rng.uniform(-1, 1, (2000, 512)).astype(np.float32)
    w = rng.uniform(-1, 1, (1100, 512)).astype(np.float32)
    wb = rng.normal(size=1100).astype(np.float32)
    got = host(tcx.linear(dev(x), dev(w), dev(wb), path="tensor"))
    ref = oracle.linear(x[:256], w, wb)
    frob_ok(got[:256], ref, 512)


@pytest.mark.parametrize("shapes", [((), (2, 2)), ((2, 2), ()), ((3,), (4,)), ((2, 3, 4), (3, 4, 5)),
                                    ((2, 3, 4), (2, 5, 6)), ((0, 3, 4), (2, 4, 5)), ((0, 3, 4), (1, 5, 6))])
def test_batched_matmul_invalid_shapes(tcx, shapes):
    """test_batched_matmul.py:53-62."""
    a, b = (torch.empty(s, device="cuda") for s in shapes)
    with pytest.raises(ValueError):
        tcx.matmul(a, b)


def test_batched_matmul_rejects_dtype_even_empty(tcx):
    """test_batched_matmul.py:65-73 (int32 operands; torch bool is no CUDA operand here)."""
    for shape in [(2, 3, 3), (0, 3, 3)]:
        a = torch.ones(shape, dtype=torch.int32, device="cuda")
        b = torch.ones(shape, dtype=torch.float32, device="cuda")
        for left, right in [(a, a), (a, b), (b, a)]:
            with pytest.raises(ValueError):
                tcx.matmul(left, right)


def test_batched_matmul_rank_limit(tcx):
    """test_batched_matmul.py:119-129: 2^15 batches over 15 axes of extent 2."""
    a = torch.ones((2,) * 15 + (1, 1), device="cuda")
    b = torch.ones((1, 1), device="cuda")
    r = tcx.matmul(a, b)
    assert tuple(r.shape) == tuple(a.shape)
    np.testing.assert_array_equal(host(r).reshape(-1), np.ones(2**15, np.float32))


@pytest.mark.parametrize("m,k,n,act", [(256, 784, 512, "relu"), (128, 4096, 256, "none"), (300, 1000, 300, "silu"),
                                       (256, 1001, 259, "relu"), (1, 2048, 256, "none")])
def test_split_k_small_products(tcx, oracle, m, k, n, act):
    """Products whose 128 x 256 tiles fill few SMs split their k-blocks over CTAs; the
    partial tiles are summed in split order with bias and activation applied after."""
    rng = np.random.default_rng(m + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    got = host(tcx.matmul(dev(a), dev(b), bias=dev(bias), act=act, path="tensor"))
    ref = oracle.add(oracle.matmul(a, b), bias)
    ref = oracle.silu(ref) if act == "silu" else oracle.relu(ref) if act == "relu" else ref
    frob_ok(got, ref, k)
    np.testing.assert_allclose(got, ref, rtol=2e-4 * math.sqrt(k / 1024) + 1e-4, atol=1e-4 * math.sqrt(k))


def test_split_k_nonfinite_takes_ieee_path(tcx, oracle):
    rng = np.random.default_rng(12)
    a = rng.uniform(-1, 1, (256, 784)).astype(np.float32)
    b = rng.uniform(-1, 1, (784, 512)).astype(np.float32)
    a[5, 9] = np.inf
    b[100, 3] = np.nan
    bias = rng.normal(size=512).astype(np.float32)
    got = host(tcx.matmul(dev(a), dev(b), bias=dev(bias), act="relu", path="tensor"))
    ref = oracle.relu(oracle.add(oracle.matmul(a, b), bias))
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4, equal_nan=True)


@pytest.mark.parametrize("m,k,n", [(256, 512, 10), (1000, 1000, 1), (3, 5000, 32), (7, 0, 9), (513, 300, 17),
                                   (64, 33, 8), (2, 1, 16)])
@pytest.mark.parametrize("act", ["none", "relu", "silu"])
def test_skinny_products(tcx, oracle, m, k, n, act):
    """n <= 32 on the FFMA path: a warp per output row, lanes split k."""
    rng = np.random.default_rng(m * 3 + n)
    a = rng.normal(size=(m, k)).astype(np.float32)
    b = rng.normal(size=(k, n)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    got = host(tcx.matmul(dev(a), dev(b), bias=dev(bias), act=act, path="auto"))
    ref = oracle.add(oracle.matmul(a, b), bias)
    ref = oracle.silu(ref) if act == "silu" else oracle.relu(ref) if act == "relu" else ref
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * math.sqrt(max(k, 1)))


def test_skinny_batched_and_linear(tcx, oracle):
    rng = np.random.default_rng(13)
    a = rng.normal(size=(2, 3, 50, 70)).astype(np.float32)
    b = rng.normal(size=(3, 70, 12)).astype(np.float32)
    np.testing.assert_allclose(host(tcx.matmul(dev(a), dev(b))), oracle.matmul(a, b), rtol=1e-4, atol=1e-3)
    x = rng.normal(size=(5, 40, 300)).astype(np.float32)
    w = rng.uniform(-0.05, 0.05, (20, 300)).astype(np.float32)
    bias = rng.normal(size=20).astype(np.float32)
    frob_ok(host(tcx.linear(dev(x), dev(w), dev(bias))), oracle.linear(x, w, bias), 300)


def test_out_tensor_checked_and_filled(tcx):
    """A caller-provided `out` receives the same result as a fresh output; an `out` of the
    wrong shape or dtype, non-contiguous, or overlapping an operand is refused before any
    launch."""
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.rand(300, 200, device="cuda", generator=g)
    b = torch.rand(200, 260, device="cuda", generator=g)
    want = tcx.matmul(a, b)
    out = torch.full((300, 260), float("nan"), device="cuda")
    got = tcx.matmul(a, b, out=out)
    torch.cuda.synchronize()
    assert got is out and torch.equal(out, want)
    for bad in (torch.empty(300, 261, device="cuda"), torch.empty(300, 260, dtype=torch.float64, device="cuda"),
                torch.empty(260, 300, device="cuda").t()):
        with pytest.raises(ValueError):
            tcx.matmul(a, b, out=bad)
    sq = torch.rand(256, 256, device="cuda", generator=g)
    with pytest.raises(ValueError):
        tcx.matmul(sq, sq.clone(), out=sq)


def test_tensor_on_another_device_is_refused(tcx):
    """Kernels launch on the current device: an operand of another GPU is an error, and
    the same call under that device's guard runs."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    a = torch.ones(4, 4, device="cuda:1")
    with pytest.raises(ValueError):
        tcx.matmul(a, a)
    with torch.cuda.device(1):
        assert float(tcx.matmul(a, a)[0, 0].item()) == 4.0
