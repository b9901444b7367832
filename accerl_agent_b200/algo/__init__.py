from .advantages import compute_gae, grpo_group_advantages, token_level_returns
from .objectives import ObjectiveConfig, padded_loss, token_objective, varlen_token_sum_loss
from .packing import (
    make_padded_collate,
    make_varlen_batch,
    padded_to_varlen,
    prepare_rl_sample,
    select_varlen_pack,
    version_lag_stats,
)
from .schedule import warmup_cosine_lr

__all__ = [
    "ObjectiveConfig",
    "compute_gae",
    "grpo_group_advantages",
    "make_padded_collate",
    "make_varlen_batch",
    "padded_loss",
    "padded_to_varlen",
    "prepare_rl_sample",
    "select_varlen_pack",
    "token_level_returns",
    "token_objective",
    "varlen_token_sum_loss",
    "version_lag_stats",
    "warmup_cosine_lr",
]
