"""Adapter training (plain-PyTorch autograd forward over the frozen model)."""
from .forward import TrainableLoRA, train_forward  # noqa: F401
from .lora_train import (Progress, TrainParameters, evaluate, iterate_batches, load_lora_data,  # noqa: F401
                         load_lora_file, loss_fn, train)
