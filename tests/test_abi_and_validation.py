"""CPU checks: the C-ABI library loads and exports every declared entry point; the host layer
validates arguments like diffrast does and refuses CPU tensors (no CPU fallback)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

import diffrast_b200 as dr
from diffrast_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "diffrast_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(dr_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.LIBRARY))
    names = declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_native.symbols())


def test_status_strings_and_version():
    lib = _native.lib()
    assert lib.dr_version() >= 1
    assert lib.dr_status_string(0).decode() == "success"
    assert "workspace" in lib.dr_status_string(10002).decode()
    with pytest.raises(RuntimeError, match="dr_raster_setup failed with status 10001"):
        _native.check(10001, "dr_raster_setup")


def test_invalid_arguments_are_rejected_without_a_gpu():
    lib = _native.lib()
    # Negative sizes and null pointers fail validation before any CUDA call.
    assert lib.dr_raster_setup(None, 1, None, -1, 0, 0, None, None, 0, 4, 4, None, None, None, 0, 0,
                               None, 0, None) == 10001
    # pos_batch must be 1 or the view count; range mode needs its prefix table.
    pos = ctypes.c_void_p(16)
    assert lib.dr_raster_setup(pos, 3, pos, 2, 3, 1, None, None, 0, 4, 4, None, pos, pos, 1 << 20,
                               1024, None, 0, None) == 10001
    assert lib.dr_raster_setup(pos, 1, pos, 2, 3, 1, pos, None, 1, 4, 4, None, pos, pos, 1 << 20,
                               1024, None, 0, None) == 10001
    # An occlusion workspace too small for the items is refused before any launch.
    assert lib.dr_raster_setup(pos, 2, pos, 2, 3, 1, None, None, 0, 4, 4, None, pos, pos, 1 << 20,
                               1024, pos, 16, None) == 10002
    assert lib.dr_raster_occlusion_workspace_bytes(1000, 2, 64, 64) >= 16000
    assert lib.dr_raster_resolve_fwd(pos, 3, pos, pos, 2, 3, 1, 4, 4, pos, pos, None) == 10001
    assert lib.dr_interpolate_fwd(None, 0, 0, 1, 0, None, None, None, 0, None, 0, 1, 1, 1, None, None, None) == 10001
    assert lib.dr_edge_neighbours(None, -5, None, None, 0, None) == 10001
    assert lib.dr_raster_setup_workspace_bytes(1000, 64, 64) >= 20000
    assert lib.dr_edge_neighbours_workspace_bytes(100) > 0


def test_cpu_tensors_are_refused():
    ctx = dr.RasterizeContext("cpu")
    pos = torch.tensor([[[-0.5, -0.5, 0.0, 1.0], [0.5, -0.5, 0.0, 1.0], [0.0, 0.5, 0.0, 1.0]]])
    tri = torch.tensor([[0, 1, 2]], dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        dr.rasterize(ctx, pos, tri, (8, 8))


@pytest.mark.parametrize(
    "call, error, pattern",
    [
        (lambda c, p, t: dr.rasterize(c, p[0, :, :3], t, (4, 4)), ValueError, r"pos must have shape"),
        (lambda c, p, t: dr.rasterize(c, p, t.long(), (4, 4)), TypeError, r"tri must be torch.int32"),
        (lambda c, p, t: dr.rasterize(c, p, t + 5, (4, 4)), ValueError, r"refers to vertex 7"),
        (lambda c, p, t: dr.rasterize(c, p, t, (0, 4)), ValueError, r"resolution must be positive"),
        (lambda c, p, t: dr.rasterize(c, p, t, "ab"), ValueError, r"resolution must be \(height, width\)"),
        (lambda c, p, t: dr.rasterize(c, p[0], t, (4, 4)), ValueError, r"ranges is required"),
        (lambda c, p, t: dr.rasterize(c, p[0], t, (4, 4), ranges=torch.tensor([[0, 2]], dtype=torch.int32)),
         ValueError, r"does not lie within"),
    ],
)
def test_rasterize_validation(call, error, pattern):
    ctx = dr.RasterizeContext("cpu")
    pos = torch.tensor([[[-0.5, -0.5, 0.0, 1.0], [0.5, -0.5, 0.0, 1.0], [0.0, 0.5, 0.0, 1.0]]])
    tri = torch.tensor([[0, 1, 2]], dtype=torch.int32)
    with pytest.raises(error, match=pattern):
        call(ctx, pos, tri)


def test_too_many_triangles_rejected():
    ctx = dr.RasterizeContext("cpu")
    pos = torch.zeros(1, 3, 4)
    tri = torch.tensor([[0, 1, 2]], dtype=torch.int32).expand((1 << 24) + 1, 3)
    with pytest.raises(ValueError, match=r"at most 2\*\*24"):
        dr.rasterize(ctx, pos, tri, (4, 4))


def test_interpolate_and_texture_validation():
    rast = torch.zeros(1, 4, 4, 4)
    tri = torch.tensor([[0, 1, 2]], dtype=torch.int32)
    attr = torch.zeros(3, 2)
    with pytest.raises(ValueError, match="rast_db is required"):
        dr.interpolate(attr, rast, tri, diff_attrs="all")
    with pytest.raises(ValueError, match="out of range"):
        dr.interpolate(attr, rast, tri, rast_db=rast, diff_attrs=[5])
    with pytest.raises(TypeError, match="sequence of channel indices"):
        dr.interpolate(attr, rast, tri, rast_db=rast, diff_attrs=[0.5])
    tex = torch.zeros(1, 8, 8, 3)
    uv = torch.zeros(1, 4, 4, 2)
    with pytest.raises(ValueError, match="Unknown filter_mode"):
        dr.texture(tex, uv, filter_mode="cubic")
    with pytest.raises(ValueError, match="requires uv_da or mip_level_bias"):
        dr.texture(tex, uv, filter_mode="linear-mipmap-linear")
    with pytest.raises(ValueError, match="cube map"):
        dr.texture(torch.zeros(1, 6, 4, 4, 3), uv)
    with pytest.raises(ValueError, match="max_mip_level must be non-negative"):
        dr.texture(tex, uv, max_mip_level=-1)
    with pytest.raises(TypeError, match="mip must be a list"):
        dr.texture(tex, uv, torch.zeros(1, 4, 4, 4), mip=5)


def test_antialias_validation():
    color = torch.zeros(1, 4, 4, 3)
    rast = torch.zeros(1, 4, 5, 4)
    pos = torch.zeros(1, 3, 4)
    tri = torch.tensor([[0, 1, 2]], dtype=torch.int32)
    with pytest.raises(ValueError, match="color must match rast"):
        dr.antialias(color, rast, pos, tri)
    with pytest.raises(TypeError, match="pos_gradient_boost must be a number"):
        dr.antialias(color, torch.zeros(1, 4, 4, 4), pos, tri, pos_gradient_boost="x")


def test_contexts_and_compat():
    gl = dr.RasterizeGLContext(output_db=False, device="cpu")
    assert gl.output_db is False and "RasterizeGLContext" in repr(gl)
    with pytest.raises(TypeError, match="output_db must be a bool"):
        dr.RasterizeGLContext("cpu")
    dr.install_as_nvdiffrast()
    import nvdiffrast.torch as nv

    assert nv.rasterize is dr.rasterize
    dr.uninstall_as_nvdiffrast()
    dr.set_backend("triton")
    with pytest.raises(ValueError, match="Unknown backend"):
        dr.set_backend("opengl")
    dr.set_log_level(2)
    assert dr.get_log_level() == 2
    dr.set_log_level(1)


def test_to_clip_validation():
    p = torch.zeros(5, 3)
    m = torch.zeros(2, 4, 4)
    with pytest.raises(ValueError, match=r"positions must have shape \[vertices, 3\]"):
        dr.to_clip(torch.zeros(5, 4), m)
    with pytest.raises(ValueError, match=r"matrix must have shape \[batch, 4, 4\]"):
        dr.to_clip(p, torch.zeros(2, 3, 4))
    with pytest.raises(TypeError, match="positions must be torch.float32"):
        dr.to_clip(p.double(), m)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        dr.to_clip(p, m)


def test_antialias_mse_validation():
    color = torch.zeros(1, 4, 4, 3)
    rast = torch.zeros(1, 4, 4, 4)
    pos = torch.zeros(1, 3, 4)
    tri = torch.tensor([[0, 1, 2]], dtype=torch.int32)
    with pytest.raises(ValueError, match="target must match color"):
        dr.antialias_mse(color, rast, pos, tri, torch.zeros(1, 4, 4, 4))
    with pytest.raises(TypeError, match="scale must be a number"):
        dr.antialias_mse(color, rast, pos, tri, torch.zeros(1, 4, 4, 3), scale="x")
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        dr.antialias_mse(color, rast, pos, tri, torch.zeros(1, 4, 4, 3))


def declared_parameters() -> dict[str, list[str]]:
    """Parameter types of every function declared in the header, by name."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(dr_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text):
        params = " ".join(params.split())
        out[name] = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
    return out


def test_binding_matches_the_header_argument_by_argument():
    """Every ctypes signature has the header's argument count, and each pointer, 64-bit, 32-bit
    or float argument is bound as one: a signature that drifted from the library would pass
    arguments into the wrong registers."""
    declared = declared_parameters()
    for name, (_, argtypes) in _native._SIGNATURES.items():
        params = declared[name]
        assert len(params) == len(argtypes), name
        for param, ctype in zip(params, argtypes, strict=True):
            if "*" in param:
                expected = {ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64),
                            ctypes.POINTER(ctypes.c_uint64)}
            elif param.startswith(("int64_t", "size_t")):
                expected = {ctypes.c_int64, ctypes.c_size_t}
            elif param.startswith(("int32_t", "int ")):
                expected = {ctypes.c_int32, ctypes.c_int}
            elif param.startswith("float"):
                expected = {ctypes.c_float}
            else:
                raise AssertionError(f"{name}: unexpected parameter {param!r}")
            assert ctype in expected, (name, param, ctype)


def test_lambert_validation():
    color = torch.zeros(1, 4, 4, 3)
    with pytest.raises(ValueError, match="normal must match color"):
        dr.lambert(color, torch.zeros(1, 4, 5, 3), torch.ones(3))
    with pytest.raises(ValueError, match="light_dir must have shape"):
        dr.lambert(color, torch.zeros(1, 4, 4, 3), torch.ones(2, 3))
    with pytest.raises(TypeError, match="light_dir must be a torch.float32 tensor"):
        dr.lambert(color, torch.zeros(1, 4, 4, 3), torch.ones(3, dtype=torch.float64))
    with pytest.raises(TypeError, match="ambient must be a number"):
        dr.lambert(color, torch.zeros(1, 4, 4, 3), torch.ones(3), ambient="x")
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        dr.lambert(color, torch.zeros(1, 4, 4, 3), torch.ones(3))
