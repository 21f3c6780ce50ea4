"""Host bookkeeping of the deferred grad_fmap2 pull (ops.LookupGrads), on CPU.

The lookups of a block keep their grad_fmap2 records; LookupGrads pulls them
in passes of at most MAX_PENDING lookups that share radius and scale, and
the sink pulls whatever is left. The pull itself is replaced by a recorder
here (no GPU): these tests check which lookups each pull gets and the
accumulate flag it is given.
"""

import torch

from localcorr_b200 import _lib, ops


def _state(monkeypatch):
    calls = []

    def fake_pull(fmap1, g2, radius, levels, scale, sort_states, records, accumulate):
        calls.append((radius, scale, [int(t.item()) for t in sort_states],
                      [int(t.item()) for t in records], accumulate))

    monkeypatch.setattr(ops, "pyramid_corr_backward_fmap2_pull", fake_pull)
    st = ops.LookupGrads(torch.zeros(1, 4, 4, 8), torch.zeros(1, 64), (1, 8, 4, 4), 2)
    return st, calls


def test_twelve_pending_lookups_pull_at_once(monkeypatch):
    st, calls = _state(monkeypatch)
    for i in range(14):
        st.defer(torch.tensor(i), torch.tensor(100 + i), 4, 0.0625)
    assert len(calls) == 1 and calls[0][2] == list(range(12))
    assert calls[0][3] == [100 + i for i in range(12)]
    assert calls[0][4] == 0  # the first pull overwrites the gradient pyramid
    st.flush()
    assert len(calls) == 2 and calls[1][2] == [12, 13]
    assert calls[1][4] == _lib.ACC_FMAP2  # later pulls add
    st.flush()
    assert len(calls) == 2  # nothing pending


def test_lookups_with_other_parameters_are_pulled_apart(monkeypatch):
    st, calls = _state(monkeypatch)
    st.defer(torch.tensor(0), torch.tensor(0), 4, 0.0625)
    st.defer(torch.tensor(1), torch.tensor(1), 4, 0.0625)
    st.defer(torch.tensor(2), torch.tensor(2), 3, 0.0625)  # another radius
    assert calls == [(4, 0.0625, [0, 1], [0, 1], 0)]
    st.flush()
    assert calls[1] == (3, 0.0625, [2], [2], _lib.ACC_FMAP2)


def test_fmap1_and_fmap2_buffers_overwrite_then_add(monkeypatch):
    st, _ = _state(monkeypatch)
    g1, f1 = st.fmap1_buffer()
    assert f1 == 0 and g1.shape == (1, 4, 4, 8)
    assert st.fmap1_buffer()[1] == _lib.ACC_FMAP1
    g2, f2 = st.fmap2_buffer()
    assert f2 == 0 and g2.dtype == torch.float32 and g2.shape == (1, 64)
    _, _, flags = st.buffers()
    assert flags == _lib.ACC_FMAP1 | _lib.ACC_FMAP2
