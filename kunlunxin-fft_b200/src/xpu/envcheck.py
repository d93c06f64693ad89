"""``src.xpu.envcheck`` -> ``bfft.envcheck`` (the reference import path, served by bfft)."""
import sys

import bfft.envcheck as _impl

sys.modules[__name__] = _impl
