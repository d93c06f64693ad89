"""``src.xpu.entry`` -> ``bfft.entry`` (the reference import path, served by bfft)."""
import sys

import bfft.entry as _impl

sys.modules[__name__] = _impl
