"""qwentts_turbo_b200: B200-native (sm_100a) decode engine for Qwen3-TTS-12Hz-0.6B.

Public API mirrors the reference package ``qwentts_turbo`` (hamza1brh/qwenTTS-turbo):
``NativeTTSGenerator`` (generator.py), ``TTSMegakernelGenerator`` (megakernel_backbone.py),
``CodePredictorMegakernelGenerator`` (megakernel_code_predictor.py). The compute runs in
libqtt.so (include/qtt.h); importing the package does not load it, the first GPU call does.
"""
from .config import DEFAULT_DIMS, ModelDims
from .weights import synthetic_weights, rope_tables


def __getattr__(name):
    if name == "NativeTTSGenerator":
        from .generator import NativeTTSGenerator
        return NativeTTSGenerator
    if name == "TTSMegakernelGenerator":
        from .megakernel_backbone import TTSMegakernelGenerator
        return TTSMegakernelGenerator
    if name == "CodePredictorMegakernelGenerator":
        from .megakernel_code_predictor import CodePredictorMegakernelGenerator
        return CodePredictorMegakernelGenerator
    raise AttributeError(name)


__version__ = "0.1.0"
