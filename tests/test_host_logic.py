"""CPU checks of host-side logic that needs no GPU: the range table of native range mode, the
capacities and overflow word of graph-captured rasterization, and the caching of device tables."""

import torch

from diffrast_b200 import _kernels as K
from diffrast_b200.context import RasterizeContext


def test_range_table_prefix_sums_and_starts():
    ranges = torch.tensor([[5, 3], [0, 0], [2, 7], [9, 1]], dtype=torch.int32)
    table = K.range_table(ranges, torch.device("cpu"))
    assert table.items == 4
    assert table.total == 11
    assert table.start.dtype == torch.int32 and table.start.tolist() == [5, 0, 2, 9]
    assert table.first.dtype == torch.int64 and table.first.tolist() == [0, 3, 3, 10]


def test_range_table_single_and_empty():
    one = K.range_table(torch.tensor([[4, 6]], dtype=torch.int32), torch.device("cpu"))
    assert (one.items, one.total, one.first.tolist()) == (1, 6, [0])
    none = K.range_table(torch.zeros(0, 2, dtype=torch.int32), torch.device("cpu"))
    assert (none.items, none.total) == (0, 0)


def test_capture_overflow_word_doubles_capacities(monkeypatch):
    dev = torch.device("cpu")
    monkeypatch.setattr(K, "_overflow", {dev: torch.zeros(1, dtype=torch.int64)})
    key = (dev, 2, 100, 64, 64)
    other = (torch.device("meta"), 2, 100, 64, 64)
    monkeypatch.setattr(K, "_graph_capacity", {key: (1024, 4096), other: (7, 9)})
    ctx = RasterizeContext("cpu")
    assert not ctx.capture_overflowed()
    assert K._graph_capacity[key] == (1024, 4096)
    K._overflow[dev][0] = 1  # as a captured binning kernel would
    assert ctx.capture_overflowed()
    assert K._graph_capacity[key] == (2048, 8192)
    assert K._graph_capacity[other] == (7, 9)  # other devices untouched
    assert int(K._overflow[dev][0]) == 0
    assert not ctx.capture_overflowed()


def test_diff_table_is_cached_per_channels_and_device():
    a = K.diff_table((0, 2, 4), torch.device("cpu"))
    b = K.diff_table((0, 2, 4), torch.device("cpu"))
    assert a is b and a.tolist() == [0, 2, 4]
    assert K.diff_table((), torch.device("cpu")) is None
