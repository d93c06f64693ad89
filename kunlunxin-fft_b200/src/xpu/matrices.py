"""``src.xpu.matrices`` -> ``bfft.matrices`` (the reference import path, served by bfft)."""
import sys

import bfft.matrices as _impl

sys.modules[__name__] = _impl
