"""``src.xpu.candidates`` -> ``bfft.candidates`` (the reference import path, served by bfft)."""
import sys

import bfft.candidates as _impl

sys.modules[__name__] = _impl
