"""``src.xpu.validate`` -> ``bfft.validate`` (the reference import path, served by bfft)."""
import sys

import bfft.validate as _impl

sys.modules[__name__] = _impl
