"""need_b200 -- NEED's gated linear-recurrence scan, written for B200 (sm_100a).

``need_b200.need_kernels`` is the drop-in for the reference's ``need_kernels``
module; ``need_b200.sp`` runs the scan sharded along T over ranks;
``need_b200.abi`` binds the C ABI of ``_lib/libneed_scan.so``.
"""
from . import abi  # noqa: F401

__all__ = ["abi", "need_kernels", "sp"]
