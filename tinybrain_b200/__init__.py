"""tinybrain_b200 -- B200-native (sm_100a) backend for TinyBrain's decode hot path.

The CUDA work lives in libtinybrain_cuda.so (C ABI: include/tinybrain_cuda.h);
this package is the host-side mirror of the reference's runtime API.
"""
from ._lib import TinyBrainError, load as load_library  # noqa: F401
from .runtime import (Context, DeviceModel, GenerationConfig, KVCacheView, LinearLayerWeights,  # noqa: F401
                      ModelConfig, ModelRunner, ModelWeights, QuantizedTensor, QuantizedWeight,
                      SamplerConfig, SeededGenerator, TokenOutput, TransformerLayerWeights,
                      attention_decode, device_count, quantize)


