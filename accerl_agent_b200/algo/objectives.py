"""Policy objectives on per-token log-probabilities (fp32 PyTorch; also the oracle of the fused kernel).

Semantics follow agent_textworld.py:893-1035:

* ratio ``r = exp(lp - old_lp)`` computed in fp32 even when the model runs in bf16;
* ``ppo``  : ``min(r*A, clip(r, 1-eps, 1+eps)*A)``
* ``gipo`` : ``r*A*exp(-0.5*(log(r_detached)/sigma)^2)`` with ``r_detached`` clamped at 1e-9
* ``sapo`` : ``sigmoid(tau*(r-1))*4/tau*A`` with ``r`` clamped to [1e-6, 1e6] and ``tau = tau_pos``
  when ``A > 0`` else ``tau_neg``
* KL k3 ``r - 1 - log r`` per token.

Varlen training optimises the global token sum ``-sum(obj) + c_kl*sum(k3)``; padded training uses a
per-sample mean (GRPO) or a per-response-then-per-sample mean (PPO) plus ``c_kl*mean(k3)``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Tuple

import torch


@dataclass(frozen=True)
class ObjectiveConfig:
    clip_mode: str = "ppo"
    clip_eps: float = 0.2
    gipo_sigma: float = 1.0
    sapo_tau_pos: float = 1.0
    sapo_tau_neg: float = 2.0
    kl_coef: float = 0.0

    @property
    def mode_id(self) -> int:
        return {"ppo": 0, "gipo": 1, "sapo": 2, "none": 3}[self.clip_mode]


def token_objective(
    logprobs: torch.Tensor, old_logprobs: torch.Tensor, advantages: torch.Tensor, cfg: ObjectiveConfig
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Return ``(objective, k3, ratio)`` per token, all fp32 and differentiable w.r.t. ``logprobs``."""
    lp = logprobs.float()
    old = old_logprobs.float()
    adv = advantages.float()
    log_ratio = lp - old
    ratio = torch.exp(log_ratio)
    if cfg.clip_mode == "ppo":
        surr1 = ratio * adv
        surr2 = torch.clamp(ratio, 1.0 - cfg.clip_eps, 1.0 + cfg.clip_eps) * adv
        obj = torch.minimum(surr1, surr2)
    elif cfg.clip_mode == "gipo":
        r_det = ratio.clamp_min(1e-9).detach()
        coeff = torch.exp(-0.5 * (torch.log(r_det) / cfg.gipo_sigma) ** 2)
        obj = ratio * adv * coeff
    elif cfg.clip_mode == "sapo":
        r = ratio.clamp(1e-6, 1e6)
        tau = torch.where(
            adv > 0,
            torch.full_like(adv, cfg.sapo_tau_pos),
            torch.full_like(adv, cfg.sapo_tau_neg),
        )
        obj = torch.sigmoid(tau * (r - 1.0)) * (4.0 / tau) * adv
    elif cfg.clip_mode == "none":
        # REINFORCE-style objective without importance ratio (vllm_fsdp.py:628-638)
        obj = adv * lp
    else:
        raise ValueError(f"Unsupported clip_mode: {cfg.clip_mode}")
    k3 = ratio - 1.0 - log_ratio
    return obj, k3, ratio


def clip_count(ratio: torch.Tensor, clip_eps: float) -> torch.Tensor:
    with torch.no_grad():
        return ((ratio < 1.0 - clip_eps) | (ratio > 1.0 + clip_eps)).sum().float()


def varlen_token_sum_loss(
    logprobs: torch.Tensor, old_logprobs: torch.Tensor, advantages: torch.Tensor, cfg: ObjectiveConfig
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Return ``(loss, stats)`` with ``loss = -sum(obj) + kl_coef*sum(k3)`` and
    ``stats = float64[policy_token_sum, k3_sum, clip_count]`` (agent_textworld.py:995-1035)."""
    obj, k3, ratio = token_objective(logprobs, old_logprobs, advantages, cfg)
    policy_sum = -obj.sum()
    k3_sum = k3.sum()
    loss = policy_sum + cfg.kl_coef * k3_sum
    clips = clip_count(ratio, cfg.clip_eps) if cfg.clip_mode == "ppo" else policy_sum.new_zeros(())
    stats = torch.stack([policy_sum.detach(), k3_sum.detach(), clips]).to(torch.float64)
    return loss, stats


def aggregate_by_sample(obj: torch.Tensor, sample_idx: torch.Tensor, counts: torch.Tensor, batch_size: int):
    """Per-sample mean of the token objective (agent_textworld.py:1068-1085)."""
    sums = torch.zeros(batch_size, device=obj.device, dtype=obj.dtype)
    sums.index_add_(0, sample_idx, obj)
    return sums / counts.to(obj.dtype)


def aggregate_by_response(obj: torch.Tensor, sample_idx: torch.Tensor, response_idx: torch.Tensor, batch_size: int):
    """Mean over tokens of each response, then mean over responses of each sample
    (agent_textworld.py:1087-1151). Samples without responses are dropped."""
    stride = int(response_idx.max().item()) + 1
    group = sample_idx.long() * stride + response_idx.long()
    uniq, inverse = torch.unique(group, sorted=False, return_inverse=True)
    resp_sum = torch.zeros(uniq.numel(), device=obj.device, dtype=obj.dtype).index_add_(0, inverse, obj)
    resp_cnt = torch.zeros_like(resp_sum).index_add_(0, inverse, torch.ones_like(obj))
    resp_mean = resp_sum / resp_cnt.clamp_min(1)
    resp_sample = torch.div(uniq, stride, rounding_mode="floor").long()
    s_sum = torch.zeros(batch_size, device=obj.device, dtype=obj.dtype).index_add_(0, resp_sample, resp_mean)
    s_cnt = torch.zeros_like(s_sum).index_add_(0, resp_sample, torch.ones_like(resp_mean))
    valid = s_cnt.gt(0)
    if not bool(valid.any()):
        raise RuntimeError("No valid response groups found for RL loss.")
    return s_sum[valid] / s_cnt[valid]


def padded_loss(
    logprobs: torch.Tensor,
    old_logprobs: torch.Tensor,
    advantages: torch.Tensor,
    sample_idx: torch.Tensor,
    response_idx: torch.Tensor,
    token_counts: torch.Tensor,
    batch_size: int,
    algorithm: str,
    cfg: ObjectiveConfig,
) -> Tuple[torch.Tensor, Dict[str, float]]:
    """Padded-layout loss: per-sample (GRPO) or per-response (PPO) mean, plus ``kl_coef*mean(k3)``."""
    obj, k3, ratio = token_objective(logprobs, old_logprobs, advantages, cfg)
    if algorithm == "ppo":
        if bool(response_idx.lt(0).any()):
            raise RuntimeError("Valid response tokens must have non-negative response indices.")
        sample_obj = aggregate_by_response(obj, sample_idx, response_idx, batch_size)
    else:
        sample_obj = aggregate_by_sample(obj, sample_idx, token_counts, batch_size)
    k3_mean = k3.mean()
    loss = -sample_obj.mean() + cfg.kl_coef * k3_mean
    stats: Dict[str, float] = {"old_new_kl_k3_token_mean": float(k3_mean.item())}
    if cfg.clip_mode == "ppo":
        stats["ppo_clip_frac"] = float(clip_count(ratio, cfg.clip_eps).item() / max(ratio.numel(), 1))
    return loss, stats


def normalize_advantages(adv: torch.Tensor, eps: float) -> torch.Tensor:
    """Batch normalisation of PPO token advantages (padded only, agent_textworld.py:962-970)."""
    return (adv - adv.mean()) / (adv.std(unbiased=False) + eps)
