"""CPU tests of the host-side shell around the kernels: the per-tensor cache, the log level, the
contexts' device resolution, the module aliases and the topology object's checks and copies.
They pin the behaviour diffrast documents for the same objects (``_cache.py``, ``log.py``,
``context.py``, ``compat.py``, ``topology.py``)."""

import copy
import gc
import pickle
import sys
import types
import warnings

import pytest
import torch

import diffrast_b200 as dr
from diffrast_b200 import compat, log
from diffrast_b200._cache import TensorCache, signature
from diffrast_b200.topology import TopologyHash


def counting(fn):
    calls = []

    def compute(t):
        calls.append(1)
        return fn(t)

    return compute, calls


def test_cache_hits_until_in_place_edit():
    compute, calls = counting(lambda t: int(t.sum()))
    cache = TensorCache(compute)
    t = torch.arange(5)
    assert cache.get(t) == 10 and cache.get(t) == 10 and len(calls) == 1
    t.add_(1)  # bumps the version counter
    assert cache.get(t) == 15 and len(calls) == 2
    t[1:3].mul_(2)  # an edit through a view counts too
    assert cache.get(t) == 20 and len(calls) == 3


def test_cache_distinguishes_objects_with_equal_contents():
    compute, calls = counting(lambda t: int(t.sum()))
    cache = TensorCache(compute)
    a, b = torch.ones(3), torch.ones(3)
    cache.get(a)
    cache.get(b)
    assert len(calls) == 2 and len(cache) == 2


def test_cache_drops_entry_when_tensor_is_freed():
    cache = TensorCache(lambda t: t.numel())
    t = torch.zeros(7)
    cache.get(t)
    assert len(cache) == 1
    del t
    gc.collect()
    assert len(cache) == 0


def test_cache_new_storage_is_a_miss():
    compute, calls = counting(lambda t: t.shape[0])
    cache = TensorCache(compute)
    t = torch.zeros(4)
    cache.get(t)
    t.set_(torch.zeros(6))  # same object, new storage and shape
    assert cache.get(t) == 6 and len(calls) == 2


def test_cache_evicts_least_recently_used():
    compute, calls = counting(lambda t: float(t[0]))
    cache = TensorCache(compute, max_entries=2)
    a, b, c = torch.zeros(1), torch.ones(1), torch.full((1,), 2.0)
    cache.get(a)
    cache.get(b)
    cache.get(a)  # a is now more recent than b
    cache.get(c)  # evicts b
    assert len(cache) == 2
    n = len(calls)
    cache.get(a)
    assert len(calls) == n  # still cached
    cache.get(b)
    assert len(calls) == n + 1  # was evicted
    with pytest.raises(ValueError):
        TensorCache(compute, max_entries=0)


def test_cache_inference_tensors_are_computed_each_time():
    compute, calls = counting(lambda t: t.numel())
    cache = TensorCache(compute)
    with torch.inference_mode():
        t = torch.zeros(3)
    assert signature(t) is None
    cache.get(t)
    cache.get(t)
    assert len(calls) == 2 and len(cache) == 0


def test_cache_clear():
    cache = TensorCache(lambda t: 1)
    keep = [torch.zeros(1) for _ in range(3)]
    for t in keep:
        cache.get(t)
    cache.clear()
    assert len(cache) == 0


def test_log_level():
    assert (log.INFO, log.WARNING, log.ERROR, log.FATAL) == (0, 1, 2, 3)
    before = dr.get_log_level()
    try:
        with pytest.raises(TypeError, match="level must be an int from 0 to 3"):
            dr.set_log_level(1.0)
        with pytest.raises(TypeError):
            dr.set_log_level("1")
        with pytest.raises(ValueError, match="level must be an int from 0 to 3"):
            dr.set_log_level(4)
        with pytest.raises(ValueError):
            dr.set_log_level(-1)
        dr.set_log_level(2)
        with warnings.catch_warnings():
            warnings.simplefilter("error")
            log.warn("silenced at level 2")
        dr.set_log_level(0)
        with pytest.warns(UserWarning, match="shown at level 0"):
            log.warn("shown at level 0")
    finally:
        dr.set_log_level(before)


def test_context_device_resolution():
    ctx = dr.RasterizeContext("cpu")
    assert ctx.device == torch.device("cpu") and ctx.output_db is True
    assert repr(ctx) == "RasterizeContext(device='cpu')"
    assert dr.RasterizeCudaContext is dr.RasterizeContext
    with pytest.raises(TypeError, match="device must be a torch.device, a string or a GPU index"):
        dr.RasterizeContext(1.5)
    with pytest.raises(TypeError):
        dr.RasterizeContext(True)
    with pytest.raises(ValueError, match="negative GPU index"):
        dr.RasterizeContext(-1)
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="no CUDA or ROCm device is available"):
            dr.RasterizeContext(0)
        with pytest.raises(RuntimeError):
            dr.RasterizeContext("cuda")
    gl = dr.RasterizeGLContext(output_db=False, device="cpu")
    assert gl.output_db is False and gl.mode == "automatic"
    assert repr(gl) == "RasterizeGLContext(output_db=False, device='cpu')"
    gl.set_context()
    gl.release_context()
    with pytest.raises(TypeError, match="output_db must be a bool"):
        dr.RasterizeGLContext(torch.device("cpu"))


@pytest.fixture
def clean_aliases():
    names = ("nvdiffrast", "nvdiffrast.torch", "diffrast", "diffrast.torch")
    saved = {n: sys.modules.get(n) for n in names}
    for n in names:  # another test may have imported the real package under one of these names
        sys.modules.pop(n, None)
    yield
    for alias in compat._ALIASES.values():
        alias.saved.clear()
    for n, m in saved.items():
        if m is None:
            sys.modules.pop(n, None)
        else:
            sys.modules[n] = m


def test_alias_install_and_uninstall(clean_aliases, monkeypatch):
    monkeypatch.setattr(compat, "_findable", lambda name: False)
    dr.install_as_nvdiffrast()
    dr.install_as_nvdiffrast()  # a second call does nothing
    import nvdiffrast.torch as nv

    assert nv.rasterize is dr.rasterize
    dr.uninstall_as_nvdiffrast()
    assert "nvdiffrast" not in sys.modules and "nvdiffrast.torch" not in sys.modules
    dr.install_as_diffrast()
    import diffrast

    assert diffrast.interpolate is dr.interpolate
    dr.uninstall_as_diffrast()
    assert "diffrast" not in sys.modules


def test_alias_refuses_real_package_without_force(clean_aliases, monkeypatch):
    monkeypatch.setattr(compat, "_findable", lambda name: True)
    with pytest.raises(RuntimeError, match="A nvdiffrast package is installed; pass force=True"):
        dr.install_as_nvdiffrast()
    dr.install_as_nvdiffrast(force=True)
    assert sys.modules["nvdiffrast"] is dr
    dr.uninstall_as_nvdiffrast()

    real = types.ModuleType("diffrast")
    sys.modules["diffrast"] = real
    with pytest.raises(RuntimeError, match="diffrast is already imported; pass force=True"):
        dr.install_as_diffrast()
    with pytest.warns(UserWarning, match="Replacing the imported diffrast"):
        dr.install_as_diffrast(force=True)
    assert sys.modules["diffrast"] is dr
    dr.uninstall_as_diffrast()
    assert sys.modules["diffrast"] is real  # the displaced module comes back


def test_topology_checks_and_copies():
    tri = torch.tensor([[0, 1, 2], [2, 1, 3]], dtype=torch.int32)
    nbr = torch.tensor([[-1, -1, 4], [-1, -1, 2]], dtype=torch.int64).view(2, 3)
    opp = torch.tensor([[-1, -1, 3], [-1, -1, 0]], dtype=torch.int32)
    topo = TopologyHash._from_tables(nbr, opp, tuple(tri.shape), tri.device)
    assert topo.neighbours(tri) is nbr and topo.opposite(tri) is opp
    assert repr(topo) == "TopologyHash(triangles=2, device='cpu')"
    with pytest.raises(ValueError, match=r"topology_hash was built for a tri of shape \(2, 3\)"):
        topo.neighbours(torch.zeros(3, 3, dtype=torch.int32))
    # A topology that remembers its source notices in-place edits of that tensor only.
    from diffrast_b200.topology import _Provenance

    topo._provenance = _Provenance(tri)
    other = tri.clone()
    tri[0, 0] = 3
    with pytest.raises(ValueError, match="tri was modified in place"):
        topo.neighbours(tri)
    assert topo.neighbours(other) is nbr
    for clone in (copy.copy(topo), copy.deepcopy(topo), pickle.loads(pickle.dumps(topo))):
        assert clone._provenance is None
        assert torch.equal(clone.neighbours(tri), nbr)
        assert torch.equal(clone.opposite(tri), opp)
    with pytest.raises(TypeError, match="topology_hash must come from"):
        from diffrast_b200.topology import topology_for

        topology_for(tri, object())
