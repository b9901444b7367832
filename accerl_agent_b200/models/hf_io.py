"""HF safetensors checkpoints for the fused parameter layout.

Saving writes the HF/Qwen names (``q_proj``/``k_proj``/``v_proj``, ``gate_proj``/``up_proj``,
per-expert ``experts.{e}.*`` as the published Qwen MoE checkpoints and vLLM's loader use), a
``config.json`` and, when there is more than one shard, ``model.safetensors.index.json``. Tied
embeddings store only ``model.embed_tokens.weight`` as ``save_pretrained`` does.

Every trainer rank holds the full compute copy of the parameters, so shard files are written by
different ranks in parallel (rank ``r`` writes files ``r, r+W, ...``) instead of funnelling all
tensors through rank 0. Loading accepts per-expert names and fused 3-D ``experts.gate_up_proj`` /
``experts.down_proj`` tensors.
"""

from __future__ import annotations

import json
import os
from typing import Dict, Iterator, List, Optional, Tuple

import torch

from .config import ModelConfig


def hf_items(cfg: ModelConfig, name: str, tensor: torch.Tensor) -> Iterator[Tuple[str, torch.Tensor]]:
    """Split one fused-layout parameter into its HF checkpoint tensors."""
    if name.endswith("self_attn.qkv_proj.weight") or name.endswith("self_attn.qkv_proj.bias"):
        base = name.rsplit("qkv_proj", 1)[0]
        suffix = name.rsplit(".", 1)[1]
        q, kv = cfg.q_dim, cfg.kv_dim
        yield f"{base}q_proj.{suffix}", tensor[:q]
        yield f"{base}k_proj.{suffix}", tensor[q : q + kv]
        yield f"{base}v_proj.{suffix}", tensor[q + kv :]
    elif name.endswith("mlp.gate_up_proj.weight") or name.endswith("shared_expert.gate_up_proj.weight"):
        base = name.rsplit("gate_up_proj", 1)[0]
        half = tensor.shape[0] // 2
        yield f"{base}gate_proj.weight", tensor[:half]
        yield f"{base}up_proj.weight", tensor[half:]
    elif name.endswith("mlp.experts.gate_up_proj"):
        base = name[: -len("gate_up_proj")]
        half = tensor.shape[1] // 2
        for e in range(tensor.shape[0]):
            yield f"{base}{e}.gate_proj.weight", tensor[e, :half]
            yield f"{base}{e}.up_proj.weight", tensor[e, half:]
    elif name.endswith("mlp.experts.down_proj"):
        base = name[: -len("down_proj")]
        for e in range(tensor.shape[0]):
            yield f"{base}{e}.down_proj.weight", tensor[e]
    else:
        yield name, tensor


def iter_hf_state(model) -> Iterator[Tuple[str, torch.Tensor]]:
    for name, view in model.named_parameters():
        yield from hf_items(model.cfg, name, view)


def _shard_plan(items: List[Tuple[str, torch.Tensor]], max_shard_bytes: int) -> List[List[Tuple[str, torch.Tensor]]]:
    shards: List[List[Tuple[str, torch.Tensor]]] = [[]]
    size = 0
    for name, t in items:
        nbytes = t.numel() * t.element_size()
        if shards[-1] and size + nbytes > max_shard_bytes:
            shards.append([])
            size = 0
        shards[-1].append((name, t))
        size += nbytes
    return shards


def save_hf_checkpoint(
    model,
    out_dir: str,
    rank: int = 0,
    world: int = 1,
    max_shard_bytes: int = 5 * 1024**3,
    dtype: Optional[torch.dtype] = None,
) -> List[str]:
    """Write this rank's share of the safetensors shards; rank 0 also writes config and index.
    Returns the files this rank wrote."""
    from safetensors.torch import save_file

    os.makedirs(out_dir, exist_ok=True)
    items = list(iter_hf_state(model))
    shards = _shard_plan(items, max_shard_bytes)
    n = len(shards)
    names = ["model.safetensors"] if n == 1 else [f"model-{i + 1:05d}-of-{n:05d}.safetensors" for i in range(n)]
    written = []
    for i in range(rank, n, world):
        tensors = {}
        for name, t in shards[i]:
            tt = t.detach()
            if dtype is not None:
                tt = tt.to(dtype)
            tensors[name] = tt.to("cpu", non_blocking=False).contiguous()
        save_file(tensors, os.path.join(out_dir, names[i]), metadata={"format": "pt"})
        written.append(names[i])
    if rank == 0:
        model.cfg.save(out_dir)
        if n > 1:
            weight_map = {name: names[i] for i, shard in enumerate(shards) for name, _ in shard}
            total = sum(t.numel() * t.element_size() for _, t in items)
            with open(os.path.join(out_dir, "model.safetensors.index.json"), "w", encoding="utf-8") as f:
                json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)
    return written


def read_hf_state(path: str) -> Dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    index = os.path.join(path, "model.safetensors.index.json")
    state: Dict[str, torch.Tensor] = {}
    if os.path.exists(index):
        with open(index, encoding="utf-8") as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
    else:
        files = ["model.safetensors"]
    for fname in files:
        state.update(load_file(os.path.join(path, fname)))
    return state


def load_hf_checkpoint(model, path: str, strict: bool = True) -> None:
    """Copy an HF checkpoint into the model's fused flat buffers."""
    state = read_hf_state(path)
    cfg = model.cfg
    used = set()
    with torch.no_grad():
        for name, view in model.named_parameters():
            if name.endswith("mlp.experts.gate_up_proj") and name in state:
                view.copy_(state[name].to(view.dtype))
                used.add(name)
                continue
            if name.endswith("mlp.experts.down_proj") and name in state:
                view.copy_(state[name].to(view.dtype))
                used.add(name)
                continue
            for hf_name, dst in hf_items(cfg, name, view):
                src = state.get(hf_name)
                if src is None:
                    if strict:
                        raise KeyError(f"checkpoint at {path} has no tensor {hf_name}")
                    continue
                if tuple(src.shape) != tuple(dst.shape):
                    raise ValueError(f"{hf_name}: checkpoint shape {tuple(src.shape)} != model {tuple(dst.shape)}")
                dst.copy_(src.to(dst.dtype))
                used.add(hf_name)
    if strict:
        extra = [n for n in state if n not in used and not (cfg.tie_word_embeddings and n == "lm_head.weight")]
        if extra:
            raise KeyError(f"unexpected tensors in checkpoint: {extra[:5]}")


def vllm_weight_metadata(model, trainable_only: bool = False):
    """Names / dtypes / shapes in HF checkpoint form (the reference's ``get_vllm_weight_metadata``)."""
    names, dtypes, shapes = [], [], []
    for name, view in model.named_parameters():
        if trainable_only and not model.layout.slots[name].trainable:
            continue
        for hf_name, t in hf_items(model.cfg, name, view):
            names.append(hf_name)
            dtypes.append(str(t.dtype).split(".")[-1])
            shapes.append(list(t.shape))
    return names, dtypes, shapes
