"""slam_hands_b200 -- B200-native (sm_100a) DROID-SLAM correlation hot path.

The compute lives in libdroidcorr.so (CUDA C++, C ABI in include/droidcorr.h);
this package is its host-side mirror of the slam-hands correlation interface.
"""
from ._lib import DroidCorrError, build, load  # noqa: F401
from .corr import DroidCorrelation  # noqa: F401
from . import configs  # noqa: F401

__all__ = ["DroidCorrelation", "DroidCorrError", "build", "load", "configs"]
