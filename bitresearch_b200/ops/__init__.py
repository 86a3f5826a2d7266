"""Python wrappers around the sm_100a kernels in ``bitresearch_b200._C``."""
from ._ext import ext, available  # noqa: F401
