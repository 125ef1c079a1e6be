"""Model adapters (LoRA / DoRA) and their registry."""
from .lora import LoRAConfiguration, LoRAContainer, LoRAParameters  # noqa: F401
from .registry import AdapterRegistry, load_adapter  # noqa: F401
