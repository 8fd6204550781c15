"""Host logic of partition.PushForwardGraphs, without a GPU.

The multi-GPU forward alternates two copies of the next layer's input: a rank
pushes into copy t only after the barrier of the previous exchange, which every
peer reaches only after its last read of copy t. That holds only while every
step uses the copy after the one the previous step used. The captured graphs
bake a copy into each graph, so replays and eager steps, in any mix, must keep
that alternation; these tests run the bookkeeping with fake graph objects.
"""
import pytest
import torch

from gnn_cuda_b200 import partition


class _Exchange:
    def __init__(self, turn: int):
        self.turn = turn


def _fakes(monkeypatch, ex, used):
    class FakeGraph:
        def __init__(self):
            self.copy = None

        def replay(self):
            used.append(self.copy)

    class FakeCapture:
        def __init__(self, g, **kw):
            assert kw.get("capture_error_mode") == "thread_local"
            self.g = g

        def __enter__(self):
            self.g.copy = ex.turn  # the copy the captured step writes and pushes
            return self

        def __exit__(self, *exc):
            return False

    monkeypatch.setattr(torch.cuda, "CUDAGraph", FakeGraph)
    monkeypatch.setattr(torch.cuda, "graph", FakeCapture)


@pytest.mark.parametrize("first_turn", [0, 1])
def test_replays_and_eager_steps_alternate_the_copies(monkeypatch, first_turn):
    ex = _Exchange(first_turn)
    used: list = []
    _fakes(monkeypatch, ex, used)

    def eager_step():
        used.append(ex.turn)
        ex.turn ^= 1  # finish(): the exchange moves to the other copy
        return "rows"

    capturing = []

    def step_during_capture():
        capturing.append(ex.turn)
        ex.turn ^= 1
        return "rows"

    graphs = partition.PushForwardGraphs(step_during_capture, ex)
    assert capturing == [first_turn, first_turn ^ 1]  # one graph per copy
    assert ex.turn == first_turn and graphs.out == "rows"
    for kind in "rrerreeere":
        if kind == "r":
            assert graphs.replay() == "rows"
        else:
            eager_step()
    assert len(used) == 10
    assert all(used[i] != used[i + 1] for i in range(len(used) - 1)), used
    assert used[0] == first_turn
    graphs.close()
    assert graphs.graphs == []


def test_a_step_that_does_not_finish_one_exchange_is_refused(monkeypatch):
    ex = _Exchange(0)
    _fakes(monkeypatch, ex, [])
    with pytest.raises(RuntimeError, match="exactly one exchange"):
        partition.PushForwardGraphs(lambda: "rows", ex)  # never moves to the other copy


def test_a_failed_capture_leaves_the_exchange_on_its_first_copy(monkeypatch):
    """Ranks whose capture failed go on eagerly with the others: all from the same copy."""
    ex = _Exchange(1)
    _fakes(monkeypatch, ex, [])
    calls = []

    def step():
        calls.append(ex.turn)
        ex.turn ^= 1  # the exchange moved on before the failure
        if len(calls) == 1:  # the first capture fails after its step moved to copy 0
            raise RuntimeError("operation not permitted when stream is capturing")
        return "rows"
    with pytest.raises(RuntimeError, match="capturing"):
        partition.PushForwardGraphs(step, ex)
    assert ex.turn == 1
