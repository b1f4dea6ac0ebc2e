"""Device-side seeded generation (tcx_sm100_random, ops.randn / ops.rand_uniform).

The generator has no bit-level counterpart in the reference (tensor.cx's randn draws
with NumPy's default_rng on the host, python/tensorcx/tensor.py:485-497), so the
oracle here is the published Philox4x32-10 block function restated in C
(oracle/tcx_oracle.c), pinned below by two known answers, plus the generator's value
mapping. On the GPU: uniform values and the stream layout are bit-exact against the
oracle; normal values agree within 4e-6 (the device uses the SFU log2 / rsqrt /
sincos and a series near u1 = 1, the oracle double precision); slices at offsets concatenate
to the whole stream; full-size moments hold.
"""
import ctypes

import numpy as np
import pytest

# ------------------------------------------------------------------ CPU: oracle pins


def test_philox_zero_vector_known_answer(oracle):
    # Philox4x32-10 of counter 0 and key 0 (Salmon et al.'s published test vector)
    assert oracle.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]


def test_philox_cpp26_engine_known_answer(oracle):
    # C++26 [rand.eng.philox]: the 10000th output of a default-constructed
    # std::philox4x32 (key {20111115, 0}, counter from 0, four words per block) is
    # 1955073260.
    block = 2499  # outputs 9997..10000 are block 2499's four words
    words = oracle.philox4x32_10([block, 0, 0, 0], [20111115, 0])
    assert words[3] == 1955073260


def test_oracle_stream_slices_concatenate(oracle):
    whole = oracle.random("normal", 1001, seed=7, offset=5)
    parts = [oracle.random("normal", 300, seed=7, offset=5), oracle.random("normal", 401, seed=7, offset=305),
             oracle.random("normal", 300, seed=7, offset=706)]
    assert np.concatenate(parts).tobytes() == whole.tobytes()


def test_oracle_moments(oracle):
    x = oracle.random("normal", 1 << 20, seed=3).astype(np.float64)
    assert abs(x.mean()) < 5 / 1024 and abs(x.var() - 1) < 0.01
    u = oracle.random("uniform", 1 << 20, seed=3, a=-1.0, b=1.0).astype(np.float64)
    assert u.min() >= -1 and u.max() < 1 and abs(u.mean()) < 5 / 1024 * 0.6


# ------------------------------------------------------------------ GPU: the kernel

gpu = pytest.mark.gpu


def _device(kind, count, seed, offset, a, b, shift=0):
    """tcx_sm100_random through the C ABI into a buffer starting `shift` floats into
    an allocation (shift 1..3: an output that is not 16-byte aligned)."""
    import torch
    from tensorcx_b200 import _abi
    buf = torch.full((count + shift + 4,), -123.0, device="cuda")
    out = buf[shift:shift + count]
    _abi.check(_abi.lib().tcx_sm100_random(None, _abi.RANDOM[kind], ctypes.c_void_p(out.data_ptr()), count, seed,
                                           offset, a, b))
    torch.cuda.synchronize()
    host = buf.cpu().numpy()
    assert (host[:shift] == -123.0).all() and (host[shift + count:] == -123.0).all(), "wrote outside the output"
    return host[shift:shift + count]


CASES = [(1, 0, 0), (3, 1, 1), (4096, 0, 0), (4099, 2, 3), (100003, 7, 1), (1 << 20, 0, 0),
         (12345, (1 << 40) + 3, 2)]


@gpu
@pytest.mark.parametrize("count,offset,shift", CASES)
@pytest.mark.parametrize("seed", [0, 2**64 - 1, 0x1234_5678_9ABC_DEF0])
def test_uniform_bit_exact(tcx, oracle, count, offset, shift, seed):
    got = _device("uniform", count, seed, offset, -1.0, 1.0, shift)
    want = oracle.random("uniform", count, seed, offset, -1.0, 1.0)
    assert got.tobytes() == want.tobytes()


@gpu
@pytest.mark.parametrize("count,offset,shift", CASES)
def test_normal_matches_oracle(tcx, oracle, count, offset, shift):
    got = _device("normal", count, 99, offset, 0.5, 2.0, shift)
    want = oracle.random("normal", count, 99, offset, 0.5, 2.0)
    # SFU log2 / rsqrt / sincos (with a series near u1 = 1) on the device against double
    np.testing.assert_allclose(got, want, rtol=4e-6, atol=4e-6)


@gpu
def test_shards_concatenate_to_the_whole_stream(tcx):
    import torch
    n = 3_000_017
    whole = tcx.randn((n,), seed=11)
    edges = [0, 750_001, 1_500_002, 2_250_003, n]
    parts = [tcx.randn((edges[i + 1] - edges[i],), seed=11, offset=edges[i]) for i in range(4)]
    assert torch.equal(torch.cat(parts), whole)


@gpu
def test_full_size_moments_and_samples(tcx, oracle):
    import torch
    n = 1 << 28
    x = tcx.randn((n,), seed=2024)
    xs = x.double()
    mean, var = float(xs.mean()), float(xs.var())
    assert abs(mean) < 5 / n ** 0.5 and abs(var - 1) < 1e-3
    idx = np.random.default_rng(0).integers(0, n, 256)
    host = x.cpu().numpy()
    for i in idx:
        np.testing.assert_allclose(host[i], oracle.random("normal", 1, 2024, int(i))[0], rtol=4e-6, atol=4e-6)
    u = tcx.rand_uniform((n,), -1.0, 1.0, seed=5)
    assert float(u.min()) >= -1.0 and float(u.max()) < 1.0
    assert abs(float(u.double().mean())) < 5 / n ** 0.5
    del x, xs, u
    torch.cuda.empty_cache()


@gpu
def test_generation_errors(tcx):
    from tensorcx_b200 import _abi
    lib = _abi.lib()
    assert lib.tcx_sm100_random(None, 5, None, 4, 0, 0, 0.0, 1.0) == _abi.INVALID_ARGUMENT
    assert lib.tcx_sm100_random(None, 0, None, -1, 0, 0, 0.0, 1.0) == _abi.INVALID_ARGUMENT
    assert lib.tcx_sm100_random(None, 0, None, 0, 0, 0, 0.0, 1.0) == _abi.OK  # nothing to write
    import torch
    out = torch.zeros(4, device="cuda")
    with pytest.raises(ValueError, match="standard deviation"):
        _abi.check(lib.tcx_sm100_random(None, 0, ctypes.c_void_p(out.data_ptr()), 4, 0, 0, 0.0, -1.0))
    assert float(out.abs().sum()) == 0.0  # rejected before any work: output untouched
    with pytest.raises(ValueError, match="low <= high"):
        tcx.rand_uniform((4,), 1.0, -1.0, seed=1)
    with pytest.raises(ValueError, match="finite"):
        tcx.rand_uniform((4,), 0.0, float("inf"), seed=1)
    with pytest.raises(ValueError, match="randn only supports float32"):
        tcx.randn((4,), dtype="int32", seed=1)
    with pytest.raises(ValueError, match="non-negative"):
        tcx.randn((-1,), seed=1)
    with pytest.raises(ValueError, match="seed"):
        tcx.randn((4,), seed=-3)
    assert tcx.randn((0, 5), seed=1).shape == (0, 5)
