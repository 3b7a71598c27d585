"""B200-native (sm_100a) Ivonar token loop: decode step, prefill and sampler behind the reference
decoder interface. The compute path is libivonar_b200.so (include/ivonar_b200.h); see
``B200Decoder`` and ``build_decoder``."""

from ._native import KernelError
from .decoder import B200Decoder, build_decoder
from .model import ModelConfig, PackedModel, build_model, load_checkpoint

__version__ = "0.1.0"

__all__ = ["B200Decoder", "KernelError", "ModelConfig", "PackedModel", "build_decoder", "build_model", "load_checkpoint"]
