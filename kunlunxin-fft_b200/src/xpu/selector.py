"""``src.xpu.selector`` -> ``bfft.selector`` (the reference import path, served by bfft)."""
import sys

import bfft.selector as _impl

sys.modules[__name__] = _impl
