"""mamba3_b200: B200-native (sm_100a) Mamba-3 SSD hot path behind the reference's Python API.

Same public names as the reference package ``mamba3`` (mamba3/__init__.py:6-19).
Kernels live in ``libmamba3_b200.so`` (C ABI: ``include/mamba3_b200.h``); build it
with ``python -m mamba3_b200.build``.
"""

__version__ = "0.1.0"

from .mamba3 import KulaMamba, RMSNorm  # noqa: E402
from .block import KulaMambaBlock, KulaMambaLM, SwiGLU  # noqa: E402
from .ssd import SSDOutput, chunked_ssd  # noqa: E402
from .scan import ssd_scan  # noqa: E402
from .decode import GraphDecoder  # noqa: E402  (extension: CUDA-graph decode loop)
from ._lib import M3bError, check_device_errors  # noqa: E402  (status codes, device error word)

__all__ = [
    "KulaMamba",
    "KulaMambaBlock",
    "KulaMambaLM",
    "RMSNorm",
    "SwiGLU",
    "SSDOutput",
    "chunked_ssd",
    "ssd_scan",
    "GraphDecoder",
    "M3bError",
    "check_device_errors",
]
