"""Learning-rate schedule: linear warm-up then cosine decay to zero at ``total_steps``
(agent_textworld.py:534-556). Applied by the trainer before every optimizer step."""

from __future__ import annotations

import math


def warmup_cosine_lr(current_step: int, peak_lr: float, warmup_steps: int, total_steps: int, start_step: int = 0) -> float:
    if current_step < start_step:
        return 0.0
    step = current_step - start_step
    if warmup_steps > 0 and step < warmup_steps:
        return peak_lr * (step / warmup_steps)
    decay_steps = total_steps - start_step - warmup_steps
    if decay_steps <= 0:
        return peak_lr
    progress = min(max((step - warmup_steps) / decay_steps, 0.0), 1.0)
    return peak_lr * 0.5 * (1.0 + math.cos(math.pi * progress))
