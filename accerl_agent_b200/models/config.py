"""Model configurations (HF ``config.json`` compatible) and the shape presets used by the benchmarks.

Families: ``qwen2`` (dense, q/k/v bias), ``qwen2_moe`` (routed experts + a gated shared expert,
softmax-top-k router without renormalisation by default), ``qwen3`` (dense, per-head q/k RMSNorm, no
q/k/v bias) and ``qwen3_moe`` (routed experts with renormalised top-k, q/k norm).
"""

from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional


@dataclass
class ModelConfig:
    model_type: str = "qwen2"
    vocab_size: int = 151936
    hidden_size: int = 1536
    num_hidden_layers: int = 28
    num_attention_heads: int = 12
    num_key_value_heads: int = 2
    head_dim: int = 128
    intermediate_size: int = 8960
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = True
    max_position_embeddings: int = 32768
    qkv_bias: bool = True
    qk_norm: bool = False
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    norm_topk_prob: bool = False
    decoder_sparse_step: int = 1
    mlp_only_layers: List[int] = field(default_factory=list)
    # tensor-parallel engine shards: routed experts stored on this rank and the global index of the
    # first one (None: all experts)
    local_experts: Optional[int] = None
    expert_offset: int = 0
    torch_dtype: str = "bfloat16"
    bos_token_id: int = 151643
    eos_token_id: int = 151645

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def layer_is_moe(self, layer: int) -> bool:
        if not self.is_moe or layer in self.mlp_only_layers:
            return False
        return (layer + 1) % max(self.decoder_sparse_step, 1) == 0

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    # ---------------------------------------------------------------- HF interop
    @classmethod
    def from_hf_dict(cls, d: Dict[str, Any]) -> "ModelConfig":
        mt = d.get("model_type", "qwen2")
        heads = d["num_attention_heads"]
        head_dim = d.get("head_dim") or d["hidden_size"] // heads
        cfg = cls(
            model_type=mt,
            vocab_size=d["vocab_size"],
            hidden_size=d["hidden_size"],
            num_hidden_layers=d["num_hidden_layers"],
            num_attention_heads=heads,
            num_key_value_heads=d.get("num_key_value_heads", heads),
            head_dim=head_dim,
            intermediate_size=d.get("intermediate_size", 0),
            rms_norm_eps=d.get("rms_norm_eps", 1e-6),
            rope_theta=float(d.get("rope_theta", (d.get("rope_parameters") or {}).get("rope_theta", 1e6))),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            max_position_embeddings=d.get("max_position_embeddings", 32768),
            qkv_bias=mt in ("qwen2", "qwen2_moe") or bool(d.get("attention_bias", False)),
            qk_norm=mt in ("qwen3", "qwen3_moe"),
            num_experts=d.get("num_experts", 0) or 0,
            num_experts_per_tok=d.get("num_experts_per_tok", 0) or 0,
            moe_intermediate_size=d.get("moe_intermediate_size", 0) or 0,
            shared_expert_intermediate_size=d.get("shared_expert_intermediate_size", 0) or 0,
            norm_topk_prob=bool(d.get("norm_topk_prob", mt == "qwen3_moe")),
            decoder_sparse_step=d.get("decoder_sparse_step", 1) or 1,
            mlp_only_layers=list(d.get("mlp_only_layers", []) or []),
            torch_dtype=str(d.get("torch_dtype", d.get("dtype", "bfloat16"))),
            bos_token_id=d.get("bos_token_id", 151643) or 151643,
            eos_token_id=d.get("eos_token_id", 151645) or 151645,
        )
        return cfg

    @classmethod
    def from_pretrained(cls, path: str) -> "ModelConfig":
        with open(os.path.join(path, "config.json"), encoding="utf-8") as f:
            return cls.from_hf_dict(json.load(f))

    def to_hf_dict(self) -> Dict[str, Any]:
        arch = {
            "qwen2": "Qwen2ForCausalLM",
            "qwen2_moe": "Qwen2MoeForCausalLM",
            "qwen3": "Qwen3ForCausalLM",
            "qwen3_moe": "Qwen3MoeForCausalLM",
        }[self.model_type]
        d: Dict[str, Any] = {
            "architectures": [arch],
            "model_type": self.model_type,
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "intermediate_size": self.intermediate_size,
            "rms_norm_eps": self.rms_norm_eps,
            "rope_theta": self.rope_theta,
            "tie_word_embeddings": self.tie_word_embeddings,
            "max_position_embeddings": self.max_position_embeddings,
            "hidden_act": "silu",
            "torch_dtype": self.torch_dtype,
            "bos_token_id": self.bos_token_id,
            "eos_token_id": self.eos_token_id,
            "use_cache": False,
        }
        if self.model_type.startswith("qwen3"):
            d["attention_bias"] = self.qkv_bias
        if self.is_moe:
            d.update(
                num_experts=self.num_experts,
                num_experts_per_tok=self.num_experts_per_tok,
                moe_intermediate_size=self.moe_intermediate_size,
                norm_topk_prob=self.norm_topk_prob,
                decoder_sparse_step=self.decoder_sparse_step,
                mlp_only_layers=self.mlp_only_layers,
            )
            if self.model_type == "qwen2_moe":
                d["shared_expert_intermediate_size"] = self.shared_expert_intermediate_size
        return d

    def save(self, path: str) -> None:
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "config.json"), "w", encoding="utf-8") as f:
            json.dump(self.to_hf_dict(), f, indent=2, sort_keys=True)
            f.write("\n")

    def num_parameters(self) -> int:
        from .transformer import parameter_specs

        return sum(int(_prod(shape)) for _, shape in parameter_specs(self))


def _prod(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


PRESETS: Dict[str, ModelConfig] = {
    # Tiny Qwen2-style smoke model (fp32 CPU / gloo plumbing run).
    "tiny-qwen2": ModelConfig(
        model_type="qwen2", vocab_size=4096, hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
        num_key_value_heads=2, head_dim=32, intermediate_size=384, rope_theta=1e6, tie_word_embeddings=False,
        torch_dtype="float32", bos_token_id=1, eos_token_id=2,
    ),
    # Tiny Qwen2-MoE-style smoke model: 6 routed experts top-2 plus a gated shared expert.
    "tiny-qwen2-moe": ModelConfig(
        model_type="qwen2_moe", vocab_size=4096, hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
        num_key_value_heads=2, head_dim=32, intermediate_size=384, rope_theta=1e6, tie_word_embeddings=False,
        torch_dtype="float32", bos_token_id=1, eos_token_id=2, num_experts=6, num_experts_per_tok=2,
        moe_intermediate_size=64, shared_expert_intermediate_size=96,
    ),
    # Qwen2.5-1.5B shape (tied embeddings).
    "qwen2.5-1.5b": ModelConfig(),
    # Qwen1.5-MoE-A2.7B shape: 60 routed experts top-4 + 4 shared experts worth (5632) intermediate.
    "qwen1.5-moe-a2.7b": ModelConfig(
        model_type="qwen2_moe", vocab_size=151936, hidden_size=2048, num_hidden_layers=24, num_attention_heads=16,
        num_key_value_heads=16, head_dim=128, intermediate_size=5632, tie_word_embeddings=False, num_experts=60,
        num_experts_per_tok=4, moe_intermediate_size=1408, shared_expert_intermediate_size=5632,
        norm_topk_prob=False,
    ),
    # Qwen3-8B shape.
    "qwen3-8b": ModelConfig(
        model_type="qwen3", vocab_size=151936, hidden_size=4096, num_hidden_layers=36, num_attention_heads=32,
        num_key_value_heads=8, head_dim=128, intermediate_size=12288, tie_word_embeddings=False, qkv_bias=False,
        qk_norm=True,
    ),
    # Qwen3-30B-A3B shape.
    "qwen3-30b-a3b": ModelConfig(
        model_type="qwen3_moe", vocab_size=151936, hidden_size=2048, num_hidden_layers=48, num_attention_heads=32,
        num_key_value_heads=4, head_dim=128, intermediate_size=6144, tie_word_embeddings=False, qkv_bias=False,
        qk_norm=True, num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768, norm_topk_prob=True,
    ),
}


def get_preset(name: str) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return ModelConfig(**asdict(PRESETS[name]))


def resolve_model_config(model_path: Optional[str]) -> ModelConfig:
    """A preset name (``preset:<name>`` or a bare known name) or an HF directory with config.json."""
    if model_path is None:
        return get_preset("qwen2.5-1.5b")
    name = model_path[len("preset:"):] if model_path.startswith("preset:") else model_path
    if name in PRESETS:
        return get_preset(name)
    return ModelConfig.from_pretrained(model_path)
