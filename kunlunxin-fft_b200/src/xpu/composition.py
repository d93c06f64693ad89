"""``src.xpu.composition`` -> ``bfft.composition`` (the reference import path, served by bfft)."""
import sys

import bfft.composition as _impl

sys.modules[__name__] = _impl
