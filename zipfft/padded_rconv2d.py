"""`zipfft.padded_rconv2d` as an importable submodule (see zipfft_b200.padded_rconv2d)."""
from zipfft_b200.padded_rconv2d import *  # noqa: F401,F403
from zipfft_b200.padded_rconv2d import corr, conv, get_supported_conv_configs  # noqa: F401
