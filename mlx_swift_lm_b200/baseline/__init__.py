"""Comparison builds: the same models and engine with library ops only."""
from .torch_lm import GreedyTorchSampler, TorchDecoderLM  # noqa: F401
