"""The tensor-parallel decode step's piecewise graph recorder (torch_npu_smollm._PiecewiseGraph)
on CPU, with stand-ins for CUDA graphs and the NCCL all-reduce.

Checked: a recorded step splits into one graph per stretch between all-reduces; no all-reduce
runs while recording; replay runs the graphs and the all-reduces in capture order, each
all-reduce on the buffer and group it was recorded with; the recorder is inactive once
recording ends, also after an error inside the step (whose open capture is closed); and
outside a recording ``_all_reduce`` is a plain ``torch.distributed.all_reduce``.
"""
import pytest
import torch
import torch.distributed as dist

import torch_npu_smollm as sm


class FakeGraph:
    """Records capture and replay events in a shared log instead of driving CUDA."""

    log = []
    made = []

    def __init__(self, keep_graph=False):
        self.keep_graph = keep_graph
        self.open = False
        self.index = len(FakeGraph.made)
        FakeGraph.made.append(self)

    def capture_begin(self, pool=None, capture_error_mode='global'):
        assert not self.open
        assert pool == 'pool' and capture_error_mode == 'thread_local'
        self.open = True
        FakeGraph.log.append(('begin', self.index))

    def capture_end(self):
        assert self.open
        self.open = False
        FakeGraph.log.append(('end', self.index))

    def replay(self):
        assert not self.open
        FakeGraph.log.append(('replay', self.index))


@pytest.fixture()
def fakes(monkeypatch):
    FakeGraph.log, FakeGraph.made = [], []
    monkeypatch.setattr(torch.cuda, 'CUDAGraph', FakeGraph)
    monkeypatch.setattr(torch.cuda, 'graph_pool_handle', lambda: 'pool')

    def all_reduce(buf, group=None):
        FakeGraph.log.append(('all_reduce', id(buf), group))

    monkeypatch.setattr(dist, 'all_reduce', all_reduce)
    yield FakeGraph.log
    sm._PiecewiseGraph.active = None


def test_step_splits_at_all_reduces_and_replays_in_order(fakes):
    o_buf, down_buf = torch.zeros(4), torch.zeros(4)

    def step():
        fakes.append(('kernels', 'attention'))
        sm._all_reduce(o_buf, 'tp')
        fakes.append(('kernels', 'mlp'))
        sm._all_reduce(down_buf, 'tp')
        fakes.append(('kernels', 'head'))
        return 'logits'

    rec = sm._PiecewiseGraph()
    assert rec.record(step) == 'logits'
    assert sm._PiecewiseGraph.active is None
    assert [s[0] for s in rec.steps] == ['graph', 'all_reduce', 'graph', 'all_reduce', 'graph']
    assert rec.steps[1][1] is o_buf and rec.steps[3][1] is down_buf
    assert all(g.keep_graph for g in rec.graphs()) and len(rec.graphs()) == 3
    # while recording: captures open and close around each stretch of kernels, no all-reduce ran
    assert fakes == [('begin', 0), ('kernels', 'attention'), ('end', 0), ('begin', 1), ('kernels', 'mlp'),
                     ('end', 1), ('begin', 2), ('kernels', 'head'), ('end', 2)]
    fakes.clear()
    rec.replay()
    assert fakes == [('replay', 0), ('all_reduce', id(o_buf), 'tp'), ('replay', 1),
                     ('all_reduce', id(down_buf), 'tp'), ('replay', 2)]


def test_error_inside_the_step_closes_the_capture(fakes):
    def step():
        sm._all_reduce(torch.zeros(2), 'tp')
        raise RuntimeError('step failed')

    rec = sm._PiecewiseGraph()
    with pytest.raises(RuntimeError, match='step failed'):
        rec.record(step)
    assert sm._PiecewiseGraph.active is None
    assert not any(g.open for g in FakeGraph.made)
    assert not any(e[0] == 'all_reduce' for e in fakes)


def test_all_reduce_outside_a_recording_is_eager(fakes):
    buf = torch.zeros(3)
    sm._all_reduce(buf, 'tp')
    assert fakes == [('all_reduce', id(buf), 'tp')]
