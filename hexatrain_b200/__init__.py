"""HexaTrain B200: the reference's explicit training-step hot path as
hand-written CUDA for sm_100a behind its runtime seam.

Native code lives in libhexatrain_b200.so (C ABI: include/hexatrain.h); this
package is its host-side mirror of the reference's Runtime API and drivers.
"""
from ._lib import NativeLibraryError, load  # noqa: F401
from .runtime import (AdamOptimizerOutputs, LmConfig, MlpFullStepOutputs, MomentumOptimizerOutputs,  # noqa: F401
                      OptimizerConfig, Runtime, RuntimeMetrics, RuntimeOptions, TinyTransformerTrainingOutputs,
                      apply_init_stability, sample_next_token, stability_learning_rate)
