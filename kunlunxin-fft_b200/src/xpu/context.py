"""``src.xpu.context`` -> ``bfft.context`` (the reference import path, served by bfft)."""
import sys

import bfft.context as _impl

sys.modules[__name__] = _impl
