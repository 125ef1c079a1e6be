"""Op layer: every hot op is a hand-written sm_100a kernel when its inputs are
CUDA tensors (libb200kernels.so, via ctypes) and the plain-PyTorch fp32
oracle of :mod:`.reference` when they are CPU tensors."""
from . import _lib, reference  # noqa: F401
from .attention import decode_max_parts, paged_decode, paged_prefill, paged_selected_decode  # noqa: F401
from .linear import WORKSPACE, gemm, gemm_qkv_rope, row_roles  # noqa: F401
from .norm import add_layernorm, add_rmsnorm, embedding, qk_norm_rope_kv, rmsnorm, silu_mul, xielu  # noqa: F401
from .sampling import argmax, argmax_confidence, logprobs, process_logits, sample  # noqa: F401
