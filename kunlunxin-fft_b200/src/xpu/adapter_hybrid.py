"""``src.xpu.adapter_hybrid`` -> ``bfft.adapter_hybrid`` (the reference import path, served by bfft)."""
import sys

import bfft.adapter_hybrid as _impl

sys.modules[__name__] = _impl
