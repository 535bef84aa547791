"""diffrast_b200: diffrast's differentiable render path on hand-written B200 (sm_100a) kernels.

The public names are those of ``diffrast`` (``src/diffrast/__init__.py:21-41``): switching is
changing the import (``import diffrast_b200 as dr``, or ``diffrast_b200.torch``). ``to_clip`` (the
world-to-clip transform of diffrast's examples), ``antialias_mse`` (antialias with a fused
squared-error loss) and ``lambert`` (shading from interpolated normals) are additions.
"""

from diffrast_b200.backends import get_backend_name, set_backend
from diffrast_b200.compat import (
    install_as_diffrast,
    install_as_nvdiffrast,
    uninstall_as_diffrast,
    uninstall_as_nvdiffrast,
)
from diffrast_b200.context import RasterizeContext, RasterizeCudaContext, RasterizeGLContext
from diffrast_b200.log import get_log_level, set_log_level
from diffrast_b200.ops import (
    MipStack,
    antialias,
    antialias_construct_topology_hash,
    antialias_mse,
    interpolate,
    lambert,
    rasterize,
    texture,
    texture_construct_mip,
    to_clip,
)
from diffrast_b200.peeling import DepthPeeler
from diffrast_b200.topology import TopologyHash

__version__ = "0.1.0"

__all__ = [
    "DepthPeeler",
    "MipStack",
    "RasterizeContext",
    "RasterizeCudaContext",
    "RasterizeGLContext",
    "TopologyHash",
    "__version__",
    "antialias",
    "antialias_construct_topology_hash",
    "antialias_mse",
    "get_backend_name",
    "get_log_level",
    "install_as_diffrast",
    "install_as_nvdiffrast",
    "interpolate",
    "lambert",
    "rasterize",
    "set_backend",
    "set_log_level",
    "texture",
    "texture_construct_mip",
    "to_clip",
    "uninstall_as_diffrast",
    "uninstall_as_nvdiffrast",
]
