"""``src.xpu.ledger`` -> ``bfft.ledger`` (the reference import path, served by bfft)."""
import sys

import bfft.ledger as _impl

sys.modules[__name__] = _impl
