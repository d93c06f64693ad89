"""``src.xpu.error_metric`` -> ``bfft.error_metric`` (the reference import path, served by bfft)."""
import sys

import bfft.error_metric as _impl

sys.modules[__name__] = _impl
