"""gsplat_core -- B200 (sm_100a) drop-in for gsplat-mlx's ``gsplat_core``
package (python_package/gsplat_core/__init__.py re-exports the nanobind
module ``_gsplat_core``; this package does the same with a ctypes binding of
``libgsplat_b200.so``).

    from gsplat_core import projection_ewa_3dgs_fused_forward, ...

Extras beyond the reference surface live in submodules: ``autograd``
(torch.autograd wiring of the operators' VJPs), ``pipeline`` (preallocated
fused training step), ``synthetic`` (seeded benchmark scenes).
"""
from ._gsplat_core import *  # noqa: F401,F403
from ._gsplat_core import (floor_log2_plus_one, intersect_tile_count,  # noqa: F401
                           intersect_tile_culled_forward, intersect_tile_encode,
                           intersect_tile_offsets, intersect_tile_sort)
from ._lib import GsplatError, LIB_PATH, load  # noqa: F401
