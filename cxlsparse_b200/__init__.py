"""B200-native NSA generative-recommendation selected-block path.

Host-side mirror of the reference plugin surface (transport backend, planner
adapters, attention-branch ops, backing pool) over the sm_100a kernels in
``libcxlsparse_b200.so`` (C ABI: ``include/cxlsparse.h``).
"""

from ._lib import CapacityError, CxsError  # noqa: F401

__all__ = ["CapacityError", "CxsError"]
