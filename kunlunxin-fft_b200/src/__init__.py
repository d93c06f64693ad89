"""Drop-in import path of the reference (``src.xpu``), served by ``bfft``."""
