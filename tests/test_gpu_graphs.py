"""CUDA-graph capture of op sequences (tensorcx_b200.graphs.CapturedSequence): the
configs[0] MLP forward (x[256,784] @ W1 + b1 -> ReLU -> @ W2 + b2 -> softmax) replayed
from a graph must equal the eager sequence bit for bit, also after its input is
rewritten in place, and the same for a sequence with a split-K product, a row op and a
full reduction."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _mlp_tensors(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(256, 784, device="cuda", generator=g)
    w1 = (torch.rand(784, 512, device="cuda", generator=g) * 2 - 1) / 784 ** 0.5
    w2 = (torch.rand(512, 10, device="cuda", generator=g) * 2 - 1) / 512 ** 0.5
    b1 = torch.randn(512, device="cuda", generator=g) * 0.1
    b2 = torch.randn(10, device="cuda", generator=g) * 0.1
    return x, w1, b1, w2, b2


def test_mlp_graph_replay_matches_eager(tcx):
    from tensorcx_b200.graphs import CapturedSequence
    x, w1, b1, w2, b2 = _mlp_tensors(0)

    def mlp():
        h = tcx.matmul(x, w1, bias=b1, act="relu")
        return tcx.softmax(tcx.matmul(h, w2, bias=b2), axis=-1)

    want = mlp().cpu().numpy()
    seq = CapturedSequence(mlp)
    try:
        got = seq().cpu().numpy()
        assert got.tobytes() == want.tobytes()
        x.copy_(torch.randn(256, 784, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5)))
        want2 = mlp().cpu().numpy()
        got2 = seq().cpu().numpy()
        assert got2.tobytes() == want2.tobytes()
        assert not np.array_equal(want, want2)
    finally:
        seq.release()


def test_graph_of_mixed_ops(tcx):
    from tensorcx_b200.graphs import CapturedSequence
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.rand(512, 512, device="cuda", generator=g) * 2 - 1
    b = torch.rand(512, 512, device="cuda", generator=g) * 2 - 1

    def seq_fn():
        c = tcx.matmul(a, b)
        return tcx.layernorm(c, axis=-1), tcx.sum(c), tcx.argmax(c, axis=1)

    want = [t.cpu().numpy() for t in seq_fn()]
    seq = CapturedSequence(seq_fn)
    try:
        for _ in range(3):
            got = [t.cpu().numpy() for t in seq()]
            for w, o in zip(want, got):
                assert o.tobytes() == w.tobytes()
    finally:
        seq.release()
