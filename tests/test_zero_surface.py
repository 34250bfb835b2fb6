"""ZeRO surface checks that need no GPU: stage validation and the stage-3
requirement of an engine-backed TransformerLM."""

import pytest

from underhfs_b200.nn import Linear
from underhfs_b200.optim import ZeroAwareAdamW, ZeroShard


def test_stage_must_be_1_2_or_3():
    with pytest.raises(ValueError, match="stage"):
        ZeroAwareAdamW(Linear(2, 2).parameters(), ZeroShard(), stage=4)


def test_stage3_needs_an_engine_transformer():
    with pytest.raises(ValueError, match="TransformerLM"):
        ZeroAwareAdamW(Linear(2, 2).parameters(), ZeroShard(0, 2), stage=3)


def test_stage3_offload_choices():
    with pytest.raises(ValueError):
        ZeroAwareAdamW(Linear(2, 2).parameters(), ZeroShard(), stage=3, offload="disk")


def test_stage_1_2_single_rank_is_plain_adamw():
    opt = ZeroAwareAdamW(Linear(2, 2).parameters(), ZeroShard(), stage=2, lr=0.1)
    assert opt.zero3 is None and opt._zero is None
