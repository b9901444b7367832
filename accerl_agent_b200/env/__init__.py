from .synthetic import SyntheticGameConfig, SyntheticTextGame, synthetic_episode_lengths
from .textworld import (
    TEXTWORLD_SYSTEM_PROMPT,
    ParsedAction,
    clean_action_text,
    format_illegal_action_feedback,
    format_initial_prompt,
    format_user_content,
    parse_model_action,
    step_reward,
    transcript_user_suffix,
)

__all__ = [
    "TEXTWORLD_SYSTEM_PROMPT",
    "ParsedAction",
    "SyntheticGameConfig",
    "SyntheticTextGame",
    "clean_action_text",
    "format_illegal_action_feedback",
    "format_initial_prompt",
    "format_user_content",
    "parse_model_action",
    "step_reward",
    "synthetic_episode_lengths",
    "transcript_user_suffix",
]
