"""objectsam_b200 — B200-native (sm_100a) convolution hot path of ObjectSAM's YOLOv8s-seg.

The compute lives in `libosam.so` (hand-written tcgen05/TMA kernels behind the C ABI of include/osam.h).
This package is the host layer above that ABI, mirroring the reference's operator interfaces.
"""
from ._lib import OsamError, lib  # noqa: F401

__version__ = "0.1.0"
