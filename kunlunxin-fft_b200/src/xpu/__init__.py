"""``src.xpu`` compatibility package: the reference's import path, served by bfft.

Code written against the reference (``from src.xpu import plan_fft``,
``from src.xpu.entry import execute_fft_plan``, ``from src.xpu.runner import
fft_dit_matrix_batch`` ...) runs unchanged on B200 with ``kunlunxin-fft_b200``
on ``sys.path``: each submodule file of this package replaces itself with the
bfft module of the same role.
"""
import bfft as _bfft
from bfft import *  # noqa: F401,F403


def __getattr__(name):
    return getattr(_bfft, name)
