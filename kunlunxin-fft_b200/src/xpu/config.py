"""``src.xpu.config`` -> ``bfft.config`` (the reference import path, served by bfft)."""
import sys

import bfft.config as _impl

sys.modules[__name__] = _impl
