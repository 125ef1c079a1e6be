"""mlx_swift_lm_b200: a Blackwell-native LLM inference and serving framework.

Hot ops are hand-written sm_100a CUDA kernels (``csrc/kernels``, loaded from
``_lib/libb200kernels.so``); the host runtime (page pool, block hashing, ...)
is native C++ (``csrc/host``, ``_lib/_b200host*.so``); the framework layer
(models, engine, API, server) is PyTorch.
"""
__version__ = "0.1.0"

from .models.config import DecoderConfig  # noqa: F401
from .models.decoder import DecoderLM  # noqa: F401
from .engine.types import Request, SamplingParams, Event, FinishReason  # noqa: F401
from .engine.scheduler import SchedulerConfig  # noqa: F401
from .engine.engine import EngineV2, EngineConfig  # noqa: F401
