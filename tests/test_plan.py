"""The product's host planning (tensorcx_b200.plan) agrees with the oracle's
restatement of cpp/tensorcx/core/shape.cpp, including its errors."""
import itertools

import pytest

from oracle import oracle as O
from tensorcx_b200 import plan

MATMUL = [((3,), (3,)), ((2, 3), (3,)), ((3,), (3, 4)), ((2, 3, 4), (2, 4, 5)), ((2, 3, 4), (4, 5)),
          ((3, 4), (2, 4, 5)), ((4,), (2, 4, 5)), ((2, 3, 4), (4,)), ((2, 1, 3, 4), (1, 5, 4, 6)),
          ((1, 2, 3, 4), (3, 1, 4, 5)), ((2, 1, 1, 3, 4), (1, 5, 1, 4, 2)), ((0, 3, 4), (1, 4, 2)),
          ((2, 3, 0), (1, 0, 4)), ((), (2, 2)), ((3,), (4,)), ((2, 3, 4), (3, 4, 5)), ((2 ** 62, 0), (0, 4))]


@pytest.mark.parametrize("shapes", MATMUL)
def test_matmul_plan(shapes):
    a, b = shapes
    try:
        ref = O.matmul_plan(list(a), list(b))
    except ValueError:
        with pytest.raises(ValueError):
            plan.matmul(a, b)
        return
    p = plan.matmul(a, b)
    assert (p.output_shape, p.batch_shape, p.lhs_batch_strides, p.rhs_batch_strides, p.m, p.k, p.n) == \
        (ref[0], ref[1], ref[2], ref[3], ref[4], ref[5], ref[6])


@pytest.mark.parametrize("shape", [(), (4,), (2, 3, 5), (2, 0, 3), (0, 2, 3), (3, 1, 4)])
def test_reduction_and_axis_plans(shape):
    rank = len(shape)
    for r in range(rank + 1):
        for axes in itertools.permutations(range(rank), r):
            p = plan.reduction(shape, axes)
            q = O.reduction_plan(list(shape), list(axes))
            assert (p.output_shape, p.index_metadata, p.reduction_size) == q
    for ax in range(-rank - 1, rank + 1):
        try:
            q = O.axis_dims(list(shape), ax)
        except ValueError:
            with pytest.raises(ValueError):
                plan.axis(shape, ax)
            continue
        assert plan.axis(shape, ax) == tuple(q)


@pytest.mark.parametrize("pair", [((4, 1, 6), (3, 1)), ((5,), (2, 5)), ((), (3,)), ((2, 3), (4,)), ((0, 1), (1, 5))])
def test_broadcast_plan(pair):
    a, b = pair
    try:
        q = O.broadcast_plan(list(a), list(b))
    except ValueError:
        with pytest.raises(ValueError):
            plan.broadcast(a, b)
        return
    assert plan.broadcast(a, b) == tuple(q)


@pytest.mark.parametrize("eps", [0.0, 1e-45, 1e-5, 1e30, -1.0, float("nan"), float("inf"), 1e100, 1e-100])
def test_epsilon(eps):
    try:
        q = O.checked_epsilon(eps)
    except ValueError:
        with pytest.raises(ValueError, match="epsilon"):
            plan.epsilon(eps)
        return
    assert plan.epsilon(eps) == q
