"""The bf16 native model on the GPU against the same weights run by the fp32 CPU path."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from accerl_agent_b200.algo.packing import make_varlen_batch
from accerl_agent_b200.core.sample import RLSample
from accerl_agent_b200.models.config import ModelConfig
from accerl_agent_b200.models.transformer import build_model


def small_cfg(model_type="qwen2", moe=False):
    cfg = ModelConfig(model_type=model_type, vocab_size=2048, hidden_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, intermediate_size=512,
                      tie_word_embeddings=True, qkv_bias=model_type.startswith("qwen2"),
                      qk_norm=model_type.startswith("qwen3"))
    if moe:
        cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size = 8, 2, 256
        cfg.norm_topk_prob = model_type == "qwen3_moe"
        if model_type == "qwen2_moe":
            cfg.shared_expert_intermediate_size = 256
    return cfg


def batch_of(lengths, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    samples = []
    for L in lengths:
        ids = torch.randint(0, vocab, (L,), generator=g).tolist()
        labels = [-100] * L
        for i in range(L // 3, L):
            labels[i] = ids[i]
        samples.append(RLSample("grpo", ids, [1] * L, labels, [0.0] * L, 0.0, [0.0] * L,
                                [0 if x != -100 else -1 for x in labels], [0]))
    return make_varlen_batch(samples)


@pytest.mark.parametrize("model_type,moe", [("qwen2", False), ("qwen3", False), ("qwen2_moe", True),
                                            ("qwen3_moe", True)])
def test_gpu_model_matches_cpu_fp32(model_type, moe):
    cfg = small_cfg(model_type, moe)
    gpu = build_model(cfg, "full", torch.device("cuda"), torch.bfloat16)
    gpu.init_weights(seed=5, std=0.05)
    cpu = build_model(cfg, "full", torch.device("cpu"), torch.float32)
    cpu.params.copy_(gpu.params.float().cpu())
    batch = batch_of([300, 77, 513], cfg.vocab_size)
    lp_c, ctx_c = cpu.forward_logprobs(batch, 513)
    dev_batch = {k: v.cuda() for k, v in batch.items()}
    lp_g, ctx_g = gpu.forward_logprobs(dev_batch, 513)
    err = (lp_g.cpu() - lp_c).abs()
    if moe:
        # bf16 router logits can flip a near-tie in the top-k choice for a handful of tokens
        assert err.median() < 0.02 and (err > 0.1).float().mean() < 0.05, err.max()
    else:
        assert err.max() < 0.1, err.max()
    w = torch.randn(lp_c.shape[0])
    cpu.backward_from_logprobs(w, ctx_c)
    gpu.backward_from_logprobs(w.cuda(), ctx_g)
    worst = 0.0
    for name, _ in cpu.named_parameters():
        if moe and ".mlp." in name:
            # bf16 router logits flip some top-k choices, which moves whole tokens between experts;
            # exact MoE gradients are pinned by the fp32 HF-parity test on the CPU
            continue
        gc, gg = cpu.g(name), gpu.g(name).float().cpu()
        rel = ((gg - gc).norm() / (gc.norm() + 1e-12)).item()
        worst = max(worst, rel)
        assert rel < (0.25 if moe else 0.05), (name, rel)
    if moe:
        for name, _ in gpu.named_parameters():
            assert torch.isfinite(gpu.g(name)).all(), name
