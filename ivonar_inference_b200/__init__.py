"""B200-native (sm_100a) Ivonar token loop: decode step, prefill and sampler behind the reference
decoder interface. The compute path is libivonar_b200.so (include/ivonar_b200.h); see
``B200Decoder`` (a subclass of the reference's ``StaticDecoder``) and ``build_decoder``."""

from ._native import KernelError
from .decoder import B200Decoder, build_decoder

__version__ = "0.2.0"

__all__ = ["B200Decoder", "KernelError", "build_decoder"]
