"""Pure algorithm pieces: packing, sample preparation, objectives, advantages, LR schedule."""

import math

import pytest
import torch

from accerl_agent_b200.algo.advantages import compute_gae, grpo_group_advantages, token_level_returns
from accerl_agent_b200.algo.objectives import (
    ObjectiveConfig,
    aggregate_by_response,
    aggregate_by_sample,
    padded_loss,
    token_objective,
    varlen_token_sum_loss,
)
from accerl_agent_b200.algo.packing import (
    make_padded_collate,
    make_varlen_batch,
    padded_to_varlen,
    prepare_rl_sample,
    select_varlen_pack,
    version_lag_stats,
)
from accerl_agent_b200.algo.schedule import warmup_cosine_lr
from accerl_agent_b200.core.sample import RLSample


def sample(n, targets, alg="grpo", adv=0.5, versions=(0,)):
    labels = [-100] * n
    resp = [-1] * n
    for i in targets:
        labels[i] = 100 + i
        resp[i] = 0
    return RLSample(alg, list(range(n)), [1] * n, labels, [-1.0] * n, adv, [0.0] * n, resp, list(versions))


def test_make_varlen_batch_layout():
    a, b = sample(5, [3, 4]), sample(4, [2])
    batch = make_varlen_batch([a, b])
    assert batch["input_ids"].shape == (1, 9)
    assert batch["cu_seqlens"].tolist() == [0, 5, 9]
    assert batch["cu_seqlens"].dtype == torch.int32
    assert batch["position_ids"][0].tolist() == [0, 1, 2, 3, 4, 0, 1, 2, 3]
    assert batch["sequence_ids"].tolist() == [0] * 5 + [1] * 4
    assert batch["target_indices"].tolist() == [3, 4, 7]
    assert batch["prediction_indices"].tolist() == [2, 3, 6]
    assert batch["sample_advantages"].tolist() == [0.5, 0.5]


def test_make_varlen_batch_rejects_bad_samples():
    with pytest.raises(ValueError):
        make_varlen_batch([])
    with pytest.raises(ValueError):
        make_varlen_batch([sample(1, [])])
    with pytest.raises(ValueError):
        make_varlen_batch([sample(4, [0, 1])])
    with pytest.raises(ValueError):
        make_varlen_batch([sample(4, [])])


def test_select_varlen_pack_first_fit_descending():
    pool = [sample(n, [n - 1]) for n in (5, 9, 3, 7)]
    selected, remaining = select_varlen_pack(pool, token_budget=12, max_sequences=3)
    assert [len(s.input_ids) for s in selected] == [9, 3]
    assert [len(s.input_ids) for s in remaining] == [5, 7]
    selected, _ = select_varlen_pack(pool, token_budget=100, max_sequences=2)
    assert [len(s.input_ids) for s in selected] == [9, 7]


def test_prepare_rl_sample_truncates_left_and_masks_first():
    s = sample(10, [1, 2, 8, 9])
    p = prepare_rl_sample(s, "grpo", max_length=8)
    assert len(p.input_ids) == 8 and p.input_ids[0] == 2
    assert p.labels[0] == -100 and p.old_logprobs[0] == 0.0 and p.response_indices[0] == -1
    assert prepare_rl_sample(s, "ppo", 8) is None
    assert prepare_rl_sample(sample(4, [0]), "grpo", 8) is None  # only target is the first token
    bad = sample(5, [3])
    bad.response_indices[3] = -1
    assert prepare_rl_sample(bad, "grpo", 8) is None
    short = sample(5, [3])
    short.old_logprobs = short.old_logprobs[:-1]
    assert prepare_rl_sample(short, "grpo", 8) is None


def test_padded_collate_and_varlen_view():
    collate = make_padded_collate(pad_token_id=0)
    batch = collate([sample(3, [2]), sample(5, [4])])
    assert batch["input_ids"].shape == (2, 5)
    assert batch["labels"][0].tolist() == [-100, -100, 102, -100, -100]
    assert batch["response_indices"][0, 3:].tolist() == [-1, -1]
    vb = padded_to_varlen(batch)
    assert vb["cu_seqlens"].tolist() == [0, 3, 8]
    assert vb["position_ids"][0].tolist() == [0, 1, 2, 0, 1, 2, 3, 4]


def test_version_lag():
    lag, n = version_lag_stats([sample(3, [2], versions=(0, 2)), sample(3, [2], versions=(5,))], 3.0)
    assert lag == 1.0 and n == 2


@pytest.mark.parametrize("mode", ["ppo", "gipo", "sapo"])
def test_token_objective_values(mode):
    lp = torch.tensor([-1.0, -2.0, -0.5, -3.0])
    old = torch.tensor([-1.5, -1.0, -0.5, -2.0])
    adv = torch.tensor([1.0, -1.0, 2.0, 0.5])
    cfg = ObjectiveConfig(clip_mode=mode, clip_eps=0.2, gipo_sigma=1.0, sapo_tau_pos=1.0, sapo_tau_neg=2.0)
    obj, k3, ratio = token_objective(lp, old, adv, cfg)
    r = torch.exp(lp - old)
    if mode == "ppo":
        want = torch.minimum(r * adv, r.clamp(0.8, 1.2) * adv)
    elif mode == "gipo":
        want = r * adv * torch.exp(-0.5 * torch.log(r) ** 2)
    else:
        tau = torch.where(adv > 0, torch.tensor(1.0), torch.tensor(2.0))
        want = torch.sigmoid(tau * (r - 1)) * 4 / tau * adv
    assert torch.allclose(obj, want)
    assert torch.allclose(k3, r - 1 - (lp - old))


def test_varlen_loss_is_token_sum():
    lp = torch.tensor([-1.0, -2.0, -0.4], requires_grad=True)
    old = torch.tensor([-1.1, -1.0, -0.5])
    adv = torch.tensor([1.0, -1.0, 2.0])
    cfg = ObjectiveConfig(kl_coef=0.1)
    loss, stats = varlen_token_sum_loss(lp, old, adv, cfg)
    obj, k3, r = token_objective(lp, old, adv, cfg)
    assert torch.allclose(loss, -obj.sum() + 0.1 * k3.sum())
    assert stats.dtype == torch.float64
    assert stats[2].item() == float(((r < 0.8) | (r > 1.2)).sum())


def test_aggregations():
    obj = torch.tensor([1.0, 3.0, 2.0, 4.0, 6.0])
    sid = torch.tensor([0, 0, 1, 1, 1])
    assert aggregate_by_sample(obj, sid, torch.tensor([2, 3]), 2).tolist() == [2.0, 4.0]
    rid = torch.tensor([0, 1, 0, 0, 1])
    # sample 0: responses {1},{3} -> mean 2 ; sample 1: responses {2,4} (3), {6} -> mean 4.5
    assert aggregate_by_response(obj, sid, rid, 2).tolist() == [2.0, 4.5]


def test_padded_loss_grpo_per_sample_mean():
    lp = torch.tensor([-1.0, -1.0, -1.0], requires_grad=True)
    old = lp.detach().clone()
    adv = torch.tensor([1.0, 1.0, -2.0])
    loss, stats = padded_loss(lp, old, adv, torch.tensor([0, 0, 1]), torch.tensor([0, 0, 0]), torch.tensor([2, 1]),
                              2, "grpo", ObjectiveConfig())
    assert math.isclose(loss.item(), -((1.0 + -2.0) / 2), rel_tol=1e-6)
    assert stats["ppo_clip_frac"] == 0.0


def test_advantages():
    labels = [-100, 5, 6, -100, 7]
    rewards = [0.0, 0.0, 1.0, 0.0, 2.0]
    assert token_level_returns(labels, rewards, 0.5) == [0.0, 1.0, 2.0, 0.0, 2.0]
    mean, std, adv = grpo_group_advantages([1.0, 0.0, 0.0, 1.0], 1e-8)
    assert mean == 0.5 and math.isclose(std, 0.5)
    assert [round(a, 6) for a in adv] == [1.0, -1.0, -1.0, 1.0]
    assert grpo_group_advantages([3.0], 1e-8)[2] == [0.0]
    assert grpo_group_advantages([1.0, 1.0], 1e-8)[2] == [0.0, 0.0]
    gae, deltas = compute_gae(torch.tensor([1.0, 1.0, 1.0]), torch.tensor([0.5, 0.6, 0.7]), gamma=0.99,
                              gae_lambda=0.95)
    assert torch.allclose(deltas, torch.tensor([1 + 0.99 * 0.6 - 0.5, 1 + 0.99 * 0.7 - 0.6, 1 - 0.7]))
    assert math.isclose(gae[2].item(), 0.3, rel_tol=1e-6)


def test_lr_schedule():
    assert warmup_cosine_lr(0, 1.0, 10, 100) == 0.0
    assert warmup_cosine_lr(5, 1.0, 10, 100) == 0.5
    assert math.isclose(warmup_cosine_lr(10, 1.0, 10, 100), 1.0)
    assert math.isclose(warmup_cosine_lr(55, 1.0, 10, 100), 0.5, rel_tol=1e-9)
    assert math.isclose(warmup_cosine_lr(100, 1.0, 10, 100), 0.0, abs_tol=1e-12)
    assert warmup_cosine_lr(3, 2.0, 0, 0) == 2.0


def test_device_padded_layout_matches_host_layout():
    """The sync-free expert layout (computed with device ops, here on CPU) places every (token, slot)
    pair in the same padded segment row as the host layout, marks tiles past the end with -1 and sends
    pairs of experts outside a tensor-parallel shard's range to the spare row."""
    import torch

    from accerl_agent_b200.models.moe import SEG, _expert_segments, device_padded_layout, padded_layout

    g = torch.Generator().manual_seed(3)
    E, k, T = 12, 4, 300
    topi = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    for lo, El in ((0, E), (4, 5)):
        order, rows, valid, lay = device_padded_layout(topi, E, lo, El)
        o_ref, counts, bounds = _expert_segments(topi, E)
        assert torch.equal(order, o_ref)
        ref = padded_layout(counts[lo : lo + El].tolist(), torch.device("cpu"))
        n_tiles_ref = ref["tile_expert"].numel()
        assert torch.equal(lay["tile_expert"][:n_tiles_ref], ref["tile_expert"])
        assert bool((lay["tile_expert"][n_tiles_ref:] == -1).all())
        assert lay["total"] % SEG == 0 and lay["total"] >= ref["total"]
        assert torch.equal(lay["row_start"], ref["row_start"]) and torch.equal(lay["rows"], ref["rows"])
        e_sorted = topi.reshape(-1)[order]
        for j in range(order.numel()):
            e = int(e_sorted[j])
            if lo <= e < lo + El:
                assert bool(valid[j])
                assert int(rows[j]) == ref["starts"][e - lo] + j - bounds[e]
            else:
                assert not bool(valid[j]) and int(rows[j]) == lay["total"]
