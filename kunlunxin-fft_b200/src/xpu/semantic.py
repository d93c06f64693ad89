"""``src.xpu.semantic`` -> ``bfft.semantic`` (the reference import path, served by bfft)."""
import sys

import bfft.semantic as _impl

sys.modules[__name__] = _impl
