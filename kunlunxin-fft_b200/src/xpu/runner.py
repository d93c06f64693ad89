"""``src.xpu.runner`` -> ``bfft.runner`` (the reference import path, served by bfft)."""
import sys

import bfft.runner as _impl

sys.modules[__name__] = _impl
