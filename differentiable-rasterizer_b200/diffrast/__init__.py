"""B200 (sm_100a) drop-in for the reference's differentiable soft-triangle rasterizer.

``diffrast.torch_layer`` mirrors the reference's torch op module; ``diffrast_rs``
(one directory up) mirrors its PyO3 extension. Both call the C ABI of
``libdiffrast_cuda.so`` (include/diffrast_cuda.h) through ``diffrast._native``.
"""

from . import _native  # noqa: F401
