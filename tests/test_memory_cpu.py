"""HBM budget policies and tickets (no device needed)."""
import pytest
import torch

from mlx_swift_lm_b200 import DecoderLM
from mlx_swift_lm_b200.kv.memory import (BudgetPolicy, FixedPolicy, MaxPolicy, MemoryBudget, SumPolicy,
                                         model_bytes)
from mlx_swift_lm_b200.models.config import tiny_qwen3


def test_policies():
    assert SumPolicy(cap=100).limit(10, [20, 30]) == 60
    assert SumPolicy(cap=50).limit(10, [20, 30]) == 50
    assert not SumPolicy(cap=50).can_admit(10, [20], 30) and SumPolicy(cap=60).can_admit(10, [20], 30)
    assert MaxPolicy().limit(10, [5, 40]) == 40
    assert FixedPolicy(77).limit(0, [1000]) == 77 and not FixedPolicy(77).can_admit(70, [], 8)
    assert BudgetPolicy(5, cap=100).limit(10, [20]) == 35


def test_budget_tickets():
    b = MemoryBudget(SumPolicy(cap=100), baseline=40)
    with b.ticket(30):
        assert b.limit == 70
        assert b.try_acquire(40) is None  # 40 + 30 + 40 > 100
        t = b.try_acquire(20)
        assert t is not None and b.limit == 90
        b.release(t)
    assert b.limit == 40
    with pytest.raises(MemoryError):
        with b.ticket(61):
            pass


def test_model_bytes():
    m = DecoderLM(tiny_qwen3(), "cpu", torch.float32).init_random(0)
    assert model_bytes(m) == 4 * m.num_params()
