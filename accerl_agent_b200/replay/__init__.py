from .buffer import ReplayBuffer, RolloutStats

__all__ = ["ReplayBuffer", "RolloutStats"]
