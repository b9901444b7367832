"""Decoder-only causal LM (Qwen2 / Qwen2-MoE / Qwen3 / Qwen3-MoE) on the native ops.

Parameters live in flat buffers in a fused, kernel-friendly layout: ``q|k|v`` projections are one
``qkv_proj`` matrix, ``gate|up`` one ``gate_up_proj`` matrix and routed experts are stacked
``[E, 2I, H]`` / ``[E, H, I]`` tensors. ``models/hf_io.py`` maps this layout to HF checkpoint names.

Training runs an explicit layer-wise forward that saves what the backward needs, and a backward that
writes weight gradients straight into fp32 gradient buffers (wgrad GEMMs accumulate with beta=1, so
gradient accumulation over micro-batches is free). Residual adds are fused into the o_proj / down_proj
GEMM epilogues; the LM head only runs on the prediction rows of the packed batch.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .. import ops
from .config import ModelConfig

ALIGN = 64  # elements; every parameter starts on a 128-byte boundary in bf16


def parameter_specs(cfg: ModelConfig) -> List[Tuple[str, Tuple[int, ...]]]:
    H, V = cfg.hidden_size, cfg.vocab_size
    specs: List[Tuple[str, Tuple[int, ...]]] = [("model.embed_tokens.weight", (V, H))]
    for layer in range(cfg.num_hidden_layers):
        p = f"model.layers.{layer}."
        specs.append((p + "input_layernorm.weight", (H,)))
        specs.append((p + "self_attn.qkv_proj.weight", (cfg.qkv_dim, H)))
        if cfg.qkv_bias:
            specs.append((p + "self_attn.qkv_proj.bias", (cfg.qkv_dim,)))
        if cfg.qk_norm:
            specs.append((p + "self_attn.q_norm.weight", (cfg.head_dim,)))
            specs.append((p + "self_attn.k_norm.weight", (cfg.head_dim,)))
        specs.append((p + "self_attn.o_proj.weight", (H, cfg.q_dim)))
        specs.append((p + "post_attention_layernorm.weight", (H,)))
        if cfg.layer_is_moe(layer):
            E, Im = cfg.num_experts, cfg.moe_intermediate_size
            El = cfg.local_experts or E
            specs.append((p + "mlp.gate.weight", (E, H)))
            if cfg.shared_expert_intermediate_size > 0:
                # right after the router so that [router; shared gate] is one [E + 1, H] matrix
                specs.append((p + "mlp.shared_expert_gate.weight", (1, H)))
            specs.append((p + "mlp.experts.gate_up_proj", (El, 2 * Im, H)))
            specs.append((p + "mlp.experts.down_proj", (El, H, Im)))
            if cfg.shared_expert_intermediate_size > 0:
                Is = cfg.shared_expert_intermediate_size
                specs.append((p + "mlp.shared_expert.gate_up_proj.weight", (2 * Is, H)))
                specs.append((p + "mlp.shared_expert.down_proj.weight", (H, Is)))
        else:
            specs.append((p + "mlp.gate_up_proj.weight", (2 * cfg.intermediate_size, H)))
            specs.append((p + "mlp.down_proj.weight", (H, cfg.intermediate_size)))
    specs.append(("model.norm.weight", (H,)))
    if not cfg.tie_word_embeddings:
        specs.append(("lm_head.weight", (V, H)))
    return specs


def is_trainable(name: str, train_mode: str, num_layers: int) -> bool:
    """``full`` / ``lm_head`` / ``last_layer`` selection (agent_textworld.py:243-262). With tied
    embeddings the LM head is the embedding matrix, which ``lm_head`` mode then trains."""
    if train_mode == "full":
        return True
    if train_mode == "lm_head":
        return "lm_head" in name
    if train_mode == "last_layer":
        return f"model.layers.{num_layers - 1}." in name or "lm_head" in name
    raise ValueError(f"Unsupported train mode: {train_mode}")


def is_expert_param(name: str) -> bool:
    """Routed-expert tensors (stacked over experts); the router and shared expert are not."""
    return name.endswith("mlp.experts.gate_up_proj") or name.endswith("mlp.experts.down_proj")


@dataclass
class ParamSlot:
    name: str
    shape: Tuple[int, ...]
    offset: int
    numel: int
    trainable: bool
    grad_offset: int = -1


@dataclass
class ParamLayout:
    """Offsets of every parameter in two flat segments: trainable first, then frozen.

    ``experts_last`` (expert-partitioned training: each rank holds only its routed experts) orders
    the trainable segment as [replicated parameters | this rank's expert tensors]: the first
    ``replicated_numel`` elements are laid out identically on every rank (sharded and reduced by the
    optimizer), the rest is rank-local."""

    slots: Dict[str, ParamSlot]
    order: List[str]
    trainable_numel: int
    total_numel: int
    replicated_numel: int = -1

    def __post_init__(self):
        if self.replicated_numel < 0:
            self.replicated_numel = self.trainable_numel

    @classmethod
    def build(cls, cfg: ModelConfig, train_mode: str = "full", pad_to: int = 1,
              experts_last: bool = False) -> "ParamLayout":
        specs = parameter_specs(cfg)
        tied = cfg.tie_word_embeddings

        def trainable(name: str) -> bool:
            if tied and name == "model.embed_tokens.weight" and train_mode != "full":
                return True if train_mode in ("lm_head", "last_layer") else False
            return is_trainable(name, train_mode, cfg.num_hidden_layers)

        slots: Dict[str, ParamSlot] = {}
        off = 0
        q = ALIGN * max(pad_to, 1)
        replicated_numel = -1
        passes = ((True, False), (True, True), (False, None)) if experts_last else ((True, None), (False, None))
        for group, experts in passes:
            for name, shape in specs:
                if trainable(name) != group:
                    continue
                if experts is not None and is_expert_param(name) != experts:
                    continue
                n = 1
                for s in shape:
                    n *= s
                slots[name] = ParamSlot(name, tuple(shape), off, n, group)
                off += (n + ALIGN - 1) // ALIGN * ALIGN
            if group:
                off = (off + q - 1) // q * q
                if experts is False:
                    replicated_numel = off
                else:
                    trainable_numel = off
        total = (off + q - 1) // q * q
        for s in slots.values():
            if s.trainable:
                s.grad_offset = s.offset
        return cls(slots, [n for n, _ in specs], trainable_numel, total, replicated_numel)


@dataclass
class LayerCache:
    x: torch.Tensor
    h1: torch.Tensor
    rstd1: torch.Tensor
    qkv: torch.Tensor
    attn: torch.Tensor
    lse: torch.Tensor
    x2: torch.Tensor
    h2: torch.Tensor
    rstd2: torch.Tensor
    mlp: Dict[str, torch.Tensor] = field(default_factory=dict)
    qk: Dict[str, torch.Tensor] = field(default_factory=dict)


@dataclass
class ForwardCtx:
    ids: torch.Tensor
    pos: torch.Tensor
    cu: torch.Tensor
    max_seqlen: int
    layers: List[Optional[LayerCache]]
    x_final: torch.Tensor
    rstd_final: torch.Tensor
    pred_idx: torch.Tensor
    rows: torch.Tensor
    logits: torch.Tensor
    labels: torch.Tensor
    lse: torch.Tensor
    first_trainable_layer: int


class CausalLM:
    """Functional model over flat parameter / gradient buffers."""

    def __init__(self, cfg: ModelConfig, layout: ParamLayout, params: torch.Tensor, grads: Optional[torch.Tensor] = None):
        self.cfg = cfg
        self.layout = layout
        self.params = params
        self.grads = grads
        self._views: Dict[str, torch.Tensor] = {}
        self._gviews: Dict[str, torch.Tensor] = {}
        self.rebind(params, grads)
        self.first_trainable_layer = self._first_trainable_layer()
        self.gradient_checkpointing = False
        self.units = None  # layer-sharded parameters (parallel/zero3.py) bind views around each layer

    @classmethod
    def without_buffers(cls, cfg: ModelConfig, layout: "ParamLayout") -> "CausalLM":
        """A model whose views are bound unit by unit by layer-sharded parameters (no flat buffers)."""
        self = cls.__new__(cls)
        self.cfg, self.layout = cfg, layout
        self.params = self.grads = None
        self._views, self._gviews = {}, {}
        self.first_trainable_layer = 0
        self.gradient_checkpointing = False
        self.units = None
        return self

    # ---------------------------------------------------------------- parameters
    def rebind(self, params: torch.Tensor, grads: Optional[torch.Tensor]) -> None:
        self.params = params
        self.grads = grads
        self._views = {n: params[s.offset : s.offset + s.numel].view(s.shape) for n, s in self.layout.slots.items()}
        self._gviews = {}
        if grads is not None:
            for n, s in self.layout.slots.items():
                if s.trainable:
                    self._gviews[n] = grads[s.grad_offset : s.grad_offset + s.numel].view(s.shape)

    def w(self, name: str) -> torch.Tensor:
        return self._views[name]

    def g(self, name: str) -> Optional[torch.Tensor]:
        return self._gviews.get(name)

    def named_parameters(self):
        for n in self.layout.order:
            yield n, self._views[n]

    def _first_trainable_layer(self) -> int:
        for layer in range(self.cfg.num_hidden_layers):
            if self.layout.slots[f"model.layers.{layer}.input_layernorm.weight"].trainable:
                return layer
        return self.cfg.num_hidden_layers

    @property
    def lm_head_name(self) -> str:
        return "model.embed_tokens.weight" if self.cfg.tie_word_embeddings else "lm_head.weight"

    def init_weights(self, seed: int = 0, std: float = 0.02) -> None:
        """Random init (normal(0, std) matrices, unit norms, zero biases), deterministic per seed."""
        if self.units is not None:
            self.units.init_weights(seed, std)
            return
        dev = self.params.device
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        with torch.no_grad():
            for name in self.layout.order:
                self._init_param(name, self._views[name], gen, std)

    def _init_param(self, name: str, v: torch.Tensor, gen: torch.Generator, std: float) -> None:
        cfg = self.cfg
        partial = cfg.local_experts is not None and cfg.local_experts != cfg.num_experts
        dev = v.device
        if name.endswith("norm.weight") or "layernorm" in name:
            v.fill_(1.0)
        elif name.endswith(".bias"):
            v.zero_()
        elif partial and is_expert_param(name):
            # draw the whole expert stack and keep this rank's experts: every partition of the
            # experts holds exactly the values of the unpartitioned model
            full = torch.randn((cfg.num_experts,) + tuple(v.shape[1:]), generator=gen, dtype=torch.float32,
                               device=dev) * std
            v.copy_(full[cfg.expert_offset : cfg.expert_offset + v.shape[0]].to(v.dtype))
        else:
            chunk = torch.randn(v.shape, generator=gen, dtype=torch.float32, device=dev) * std
            v.copy_(chunk.to(v.dtype))

    # ---------------------------------------------------------------- forward
    def _layer_forward(self, layer: int, x: torch.Tensor, pos, cu, max_seqlen, save: bool):
        cfg = self.cfg
        p = f"model.layers.{layer}."
        H, D = cfg.hidden_size, cfg.head_dim
        Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        h1, rstd1 = ops.rmsnorm(x, self.w(p + "input_layernorm.weight"), cfg.rms_norm_eps)
        bias = self.w(p + "self_attn.qkv_proj.bias") if cfg.qkv_bias else None
        qk: Dict[str, torch.Tensor] = {}
        # the RoPE kernel computes each token's cos/sin once for all heads; the projection's fused RoPE
        # epilogue (ops.linear_rope) recomputes them per tile and measured slower in this step
        qkv = ops.linear(h1, self.w(p + "self_attn.qkv_proj.weight"), bias=bias)
        if cfg.qk_norm:
            qk = self._qk_norm_forward(layer, qkv)
        ops.rope_(qkv, pos, Hq + Hkv, D, cfg.rope_theta)
        q = qkv[:, : cfg.q_dim]
        k = qkv[:, cfg.q_dim : cfg.q_dim + cfg.kv_dim]
        v = qkv[:, cfg.q_dim + cfg.kv_dim :]
        attn, lse = ops.attention_varlen(q, k, v, cu, max_seqlen, Hq, Hkv, D)
        x2 = ops.linear(attn, self.w(p + "self_attn.o_proj.weight"), residual=x)
        h2, rstd2 = ops.rmsnorm(x2, self.w(p + "post_attention_layernorm.weight"), cfg.rms_norm_eps)
        if cfg.layer_is_moe(layer):
            from .moe import moe_forward

            x3, mlp_cache = moe_forward(self, layer, h2, x2, save)
        else:
            if save:
                # training keeps g|u for the backward: measured faster as the plain GEMM plus the
                # SwiGLU kernel (which reads g|u back from L2) than as the three-output fused epilogue
                gu = ops.linear(h2, self.w(p + "mlp.gate_up_proj.weight"))
                act = ops.swiglu(gu)
            else:
                act, gu = ops.linear_swiglu(h2, self.w(p + "mlp.gate_up_proj.weight"))
            x3 = ops.linear(act, self.w(p + "mlp.down_proj.weight"), residual=x2)
            mlp_cache = {"gu": gu, "act": act} if save else {}
        cache = LayerCache(x, h1, rstd1, qkv, attn, lse, x2, h2, rstd2, mlp_cache, qk) if save else None
        return x3, cache

    def _qk_norm_forward(self, layer: int, qkv: torch.Tensor) -> Dict[str, torch.Tensor]:
        """Per-head RMSNorm of q and k (Qwen3) applied in place; returns what the backward needs."""
        cfg = self.cfg
        p = f"model.layers.{layer}.self_attn."
        T, D = qkv.shape[0], cfg.head_dim
        Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        q_raw = qkv[:, : cfg.q_dim].reshape(T * Hq, D).clone()
        k_raw = qkv[:, cfg.q_dim : cfg.q_dim + cfg.kv_dim].reshape(T * Hkv, D).clone()
        qn, rq = ops.rmsnorm(q_raw, self.w(p + "q_norm.weight"), cfg.rms_norm_eps)
        kn, rk = ops.rmsnorm(k_raw, self.w(p + "k_norm.weight"), cfg.rms_norm_eps)
        qkv[:, : cfg.q_dim].copy_(qn.view(T, cfg.q_dim))
        qkv[:, cfg.q_dim : cfg.q_dim + cfg.kv_dim].copy_(kn.view(T, cfg.kv_dim))
        return {"q_raw": q_raw, "k_raw": k_raw, "rq": rq, "rk": rk}

    def forward_hidden(self, ids: torch.Tensor, pos: torch.Tensor, cu: torch.Tensor, max_seqlen: int, save: bool):
        units = self.units
        if units is not None:
            units.begin_forward()
        x = ops.embedding(ids, self.w("model.embed_tokens.weight"))
        caches: List[Optional[LayerCache]] = []
        start_save = self.first_trainable_layer
        for layer in range(self.cfg.num_hidden_layers):
            if units is not None:
                units.before_forward(layer)
            keep = save and layer >= start_save
            if keep and self.gradient_checkpointing:
                x_in = x
                x, _ = self._layer_forward(layer, x, pos, cu, max_seqlen, save=False)
                caches.append(LayerCache(x_in, *(None,) * 8))  # type: ignore[arg-type]
            else:
                x, cache = self._layer_forward(layer, x, pos, cu, max_seqlen, save=keep)
                caches.append(cache)
        return x, caches

    def forward_logprobs(self, batch: Dict[str, torch.Tensor], max_seqlen: int, save: bool = True,
                         with_entropy: bool = False):
        """Label log-probabilities at ``batch['target_indices']`` of a packed batch (response-only
        LM head). Returns ``(logprobs [n] fp32, ctx)``."""
        ids = batch["input_ids"].reshape(-1)
        pos = batch["position_ids"].reshape(-1)
        cu = batch["cu_seqlens"]
        pred_idx = batch["prediction_indices"]
        labels = batch["target_labels"] if "target_labels" in batch else batch["labels"][batch["target_indices"]]
        x, caches = self.forward_hidden(ids, pos, cu, max_seqlen, save)
        hN, rstdN = ops.rmsnorm(x, self.w("model.norm.weight"), self.cfg.rms_norm_eps)
        rows = hN.index_select(0, pred_idx)
        # vocabulary-chunked LM head: no [targets, vocab] logits tensor is built
        lp, lse, ent = ops.lm_head_logprobs(rows, self.w(self.lm_head_name), labels, with_entropy=with_entropy)
        ctx = ForwardCtx(ids, pos, cu, max_seqlen, caches, x, rstdN, pred_idx, rows, None, labels, lse,
                         self.first_trainable_layer)
        if with_entropy:
            ctx.entropy = ent  # type: ignore[attr-defined]
        return lp, ctx

    # ---------------------------------------------------------------- backward
    def backward_from_logprobs(self, dlp: torch.Tensor, ctx: ForwardCtx) -> None:
        cfg = self.cfg
        units = self.units
        if units is not None:
            units.begin_backward()
        W = self.w(self.lm_head_name)
        gW = self.g(self.lm_head_name)
        need_drows = not (self.first_trainable_layer >= cfg.num_hidden_layers and self.g("model.norm.weight") is None)
        drows = ops.lm_head_backward(ctx.rows, W, ctx.labels, ctx.lse, dlp.float(), gW, need_drows)
        if not need_drows:
            if units is not None:
                units.end_backward()
            return
        dhN = torch.zeros_like(ctx.x_final)
        dhN.index_copy_(0, ctx.pred_idx, drows)
        dx = ops.rmsnorm_backward(dhN, ctx.x_final, self.w("model.norm.weight"), ctx.rstd_final,
                                  dw_grad=self.g("model.norm.weight"))
        for layer in range(cfg.num_hidden_layers - 1, -1, -1):
            if layer < self.first_trainable_layer:
                break
            if units is not None:
                units.before_backward(layer)
            cache = ctx.layers[layer]
            if cache is not None and cache.h1 is None:  # gradient checkpointing: recompute this layer
                _, cache = self._layer_forward(layer, cache.x, ctx.pos, ctx.cu, ctx.max_seqlen, save=True)
            dx = self._layer_backward(layer, dx, cache, ctx)
            ctx.layers[layer] = None
            if units is not None:
                units.after_backward(layer)
        gE = self.g("model.embed_tokens.weight")
        if gE is not None and self.first_trainable_layer == 0:
            ops.embedding_backward(ctx.ids, dx, gE)
        if units is not None:
            units.end_backward()

    def _layer_backward(self, layer: int, dx3: torch.Tensor, c: LayerCache, ctx: ForwardCtx) -> torch.Tensor:
        cfg = self.cfg
        p = f"model.layers.{layer}."
        D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        if cfg.layer_is_moe(layer):
            from .moe import moe_backward

            dh2 = moe_backward(self, layer, dx3, c)
        else:
            Wd = self.w(p + "mlp.down_proj.weight")
            da = ops.linear_dgrad(dx3, Wd)
            ops.linear_wgrad(dx3, c.mlp["act"], self.g(p + "mlp.down_proj.weight"))
            dgu = ops.swiglu_backward(da, c.mlp["gu"])
            del da
            dh2 = ops.linear_dgrad(dgu, self.w(p + "mlp.gate_up_proj.weight"))
            ops.linear_wgrad(dgu, c.h2, self.g(p + "mlp.gate_up_proj.weight"))
            del dgu
        dx2 = ops.rmsnorm_backward(dh2, c.x2, self.w(p + "post_attention_layernorm.weight"), c.rstd2, dx_accum=dx3,
                                   dw_grad=self.g(p + "post_attention_layernorm.weight"))
        del dh2
        dattn = ops.linear_dgrad(dx2, self.w(p + "self_attn.o_proj.weight"))
        ops.linear_wgrad(dx2, c.attn, self.g(p + "self_attn.o_proj.weight"))
        q = c.qkv[:, : cfg.q_dim]
        k = c.qkv[:, cfg.q_dim : cfg.q_dim + cfg.kv_dim]
        v = c.qkv[:, cfg.q_dim + cfg.kv_dim :]
        dqkv = torch.empty_like(c.qkv)
        fuse_rope = dattn.is_cuda and D == 128
        ops.attention_varlen_backward(
            dattn, q, k, v, c.attn, c.lse, ctx.cu, ctx.max_seqlen, Hq, Hkv, D,
            dq=dqkv[:, : cfg.q_dim], dk=dqkv[:, cfg.q_dim : cfg.q_dim + cfg.kv_dim], dv=dqkv[:, cfg.q_dim + cfg.kv_dim :],
            rope_pos=ctx.pos.view(-1) if fuse_rope else None, rope_theta=cfg.rope_theta,
        )
        del dattn
        if not fuse_rope:
            ops.rope_(dqkv, ctx.pos, Hq + Hkv, D, cfg.rope_theta, inverse=True)
        if cfg.qk_norm:
            self._qk_norm_backward(layer, dqkv, c)
        if cfg.qkv_bias:
            ops.bias_grad(dqkv, self.g(p + "self_attn.qkv_proj.bias"))
        dh1 = ops.linear_dgrad(dqkv, self.w(p + "self_attn.qkv_proj.weight"))
        ops.linear_wgrad(dqkv, c.h1, self.g(p + "self_attn.qkv_proj.weight"))
        del dqkv
        dx = ops.rmsnorm_backward(dh1, c.x, self.w(p + "input_layernorm.weight"), c.rstd1, dx_accum=dx2,
                                  dw_grad=self.g(p + "input_layernorm.weight"))
        return dx

    def _qk_norm_backward(self, layer: int, dqkv: torch.Tensor, c: LayerCache) -> None:
        cfg = self.cfg
        p = f"model.layers.{layer}.self_attn."
        T, D = dqkv.shape[0], cfg.head_dim
        dq = dqkv[:, : cfg.q_dim].reshape(T * cfg.num_attention_heads, D).contiguous()
        dk = dqkv[:, cfg.q_dim : cfg.q_dim + cfg.kv_dim].reshape(T * cfg.num_key_value_heads, D).contiguous()
        dq_raw = ops.rmsnorm_backward(dq, c.qk["q_raw"], self.w(p + "q_norm.weight"), c.qk["rq"],
                                      dw_grad=self.g(p + "q_norm.weight"))
        dk_raw = ops.rmsnorm_backward(dk, c.qk["k_raw"], self.w(p + "k_norm.weight"), c.qk["rk"],
                                      dw_grad=self.g(p + "k_norm.weight"))
        dqkv[:, : cfg.q_dim].copy_(dq_raw.view(T, cfg.q_dim))
        dqkv[:, cfg.q_dim : cfg.q_dim + cfg.kv_dim].copy_(dk_raw.view(T, cfg.kv_dim))

    # ---------------------------------------------------------------- inference helpers
    @torch.no_grad()
    def forward_logits_full(self, ids: torch.Tensor, pos: torch.Tensor, cu: torch.Tensor, max_seqlen: int):
        """Logits of every position (tests / evaluation)."""
        x, _ = self.forward_hidden(ids.reshape(-1), pos.reshape(-1), cu, max_seqlen, save=False)
        hN, _ = ops.rmsnorm(x, self.w("model.norm.weight"), self.cfg.rms_norm_eps)
        return ops.linear(hN, self.w(self.lm_head_name))


def build_model(cfg: ModelConfig, train_mode: str, device, dtype: torch.dtype, with_grads: bool = True,
                pad_to: int = 1, experts_last: bool = False) -> CausalLM:
    layout = ParamLayout.build(cfg, train_mode, pad_to=pad_to, experts_last=experts_last)
    params = torch.zeros(layout.total_numel, dtype=dtype, device=device)
    grads = torch.zeros(layout.trainable_numel, dtype=torch.float32, device=device) if with_grads else None
    return CausalLM(cfg, layout, params, grads)
