"""aria_b200 -- B200-native (sm_100a) Q4_0 projection engine for ARIA's Efkolos decoder.

The product is libaria_q4.so (C ABI in include/aria_q4.h); this package is the
host-side mirror of the reference's call surface plus the benchmark harness
plumbing.  Importing it does not load CUDA; the first call does.
"""
from ._lib import AriaQ4Error, LAYOUT_KN, LAYOUT_NK  # noqa: F401

__version__ = "0.1.0"
