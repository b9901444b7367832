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


def _expert_offset(cfg: ModelConfig, tensor: torch.Tensor) -> int:
    return cfg.expert_offset if tensor.shape[0] != cfg.num_experts else 0


def _partitioned(cfg: ModelConfig) -> bool:
    return cfg.local_experts is not None and cfg.local_experts != cfg.num_experts


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
        # a model holding a subset of the experts (expert-partitioned training, a tensor-parallel engine
        # shard) names them by their global index
        base = name[: -len("gate_up_proj")]
        half = tensor.shape[1] // 2
        off = _expert_offset(cfg, tensor)
        for e in range(tensor.shape[0]):
            yield f"{base}{off + e}.gate_proj.weight", tensor[e, :half]
            yield f"{base}{off + e}.up_proj.weight", tensor[e, half:]
    elif name.endswith("mlp.experts.down_proj"):
        base = name[: -len("down_proj")]
        off = _expert_offset(cfg, tensor)
        for e in range(tensor.shape[0]):
            yield f"{base}{off + e}.down_proj.weight", tensor[e]
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
    Returns the files this rank wrote.

    With expert-partitioned storage the replicated tensors are sharded over the ranks as usual and
    every rank writes its own experts to ``model-experts-<rank>-of-<world>.safetensors``; rank 0's
    index names every expert's file from the (deterministic) expert ranges."""
    from safetensors.torch import save_file

    os.makedirs(out_dir, exist_ok=True)
    cfg = model.cfg
    items = list(iter_hf_state(model))
    partitioned = _partitioned(cfg)
    rep_items = [(n, t) for n, t in items if not (partitioned and ".mlp.experts." in n)]
    shards = _shard_plan(rep_items, max_shard_bytes)
    n = len(shards)
    single = n == 1 and not partitioned
    names = ["model.safetensors"] if single else [f"model-{i + 1:05d}-of-{n:05d}.safetensors" for i in range(n)]

    def _write(fname, pairs):
        tensors = {}
        for name, t in pairs:
            tt = t.detach()
            if dtype is not None:
                tt = tt.to(dtype)
            tensors[name] = tt.to("cpu", non_blocking=False).contiguous()
        save_file(tensors, os.path.join(out_dir, fname), metadata={"format": "pt"})

    written = []
    for i in range(rank, n, world):
        _write(names[i], shards[i])
        written.append(names[i])
    expert_file = lambda r: f"model-experts-{r + 1:05d}-of-{world:05d}.safetensors"  # noqa: E731
    if partitioned:
        _write(expert_file(rank), [(nm, t) for nm, t in items if ".mlp.experts." in nm])
        written.append(expert_file(rank))
    if rank == 0:
        base_cfg = cfg
        if partitioned:
            import copy

            base_cfg = copy.deepcopy(cfg)
            base_cfg.local_experts, base_cfg.expert_offset = None, 0
        base_cfg.save(out_dir)
        if not single:
            weight_map = {name: names[i] for i, shard in enumerate(shards) for name, _ in shard}
            total = sum(t.numel() * t.element_size() for _, t in rep_items)
            if partitioned:
                from ..parallel.expert_parallel import expert_ranges

                nloc, lo = expert_ranges(cfg.num_experts, world)
                owner = [r for r in range(world) for _ in range(nloc[r])]
                el = None if dtype is None else torch.empty((), dtype=dtype).element_size()
                for name, t in items:
                    if ".mlp.experts." not in name:
                        continue
                    # this rank's experts give the names and sizes; every expert id maps to its owner
                    head, rest = name.split(".mlp.experts.", 1)
                    e, tail = rest.split(".", 1)
                    for g in range(cfg.num_experts):
                        if int(e) == cfg.expert_offset:  # one pass over the local expert 0's names
                            weight_map[f"{head}.mlp.experts.{g}.{tail}"] = expert_file(owner[g])
                            total += t.numel() * (el or t.element_size())
            with open(os.path.join(out_dir, "model.safetensors.index.json"), "w", encoding="utf-8") as f:
                json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)
    return written


def read_hf_state(path: str, names=None) -> Dict[str, torch.Tensor]:
    """All tensors of a checkpoint, or only ``names`` (then only the files holding them are opened)."""
    from safetensors import safe_open
    from safetensors.torch import load_file

    index = os.path.join(path, "model.safetensors.index.json")
    state: Dict[str, torch.Tensor] = {}
    if os.path.exists(index):
        with open(index, encoding="utf-8") as f:
            wmap = json.load(f)["weight_map"]
        files = sorted(set(wmap.values()))
    else:
        wmap = None
        files = ["model.safetensors"]
    if names is None:
        for fname in files:
            state.update(load_file(os.path.join(path, fname)))
        return state
    wanted = set(names)
    if wmap is not None:
        files = sorted({wmap[n] for n in wanted if n in wmap})
    for fname in files:
        with safe_open(os.path.join(path, fname), framework="pt") as f:
            for key in f.keys():
                if key in wanted:
                    state[key] = f.get_tensor(key)
    return state


def load_hf_checkpoint(model, path: str, strict: bool = True) -> None:
    """Copy an HF checkpoint into the model's fused flat buffers. A model holding a subset of the
    experts reads only its experts (and opens only the files that hold what it needs)."""
    cfg = model.cfg
    partitioned = _partitioned(cfg)
    if partitioned:
        wanted = [hf for name, view in model.named_parameters() for hf, _ in hf_items(cfg, name, view)]
        wanted += [name for name, _ in model.named_parameters() if ".mlp.experts." in name]  # fused 3-D form
        state = read_hf_state(path, wanted)
    else:
        state = read_hf_state(path)
    used = set()
    _load_views(cfg, state, model.named_parameters(), path, strict, used)
    if strict and not partitioned:
        extra = [n for n in state if n not in used and not (cfg.tie_word_embeddings and n == "lm_head.weight")]
        if extra:
            raise KeyError(f"unexpected tensors in checkpoint: {extra[:5]}")


def _load_views(cfg: ModelConfig, state, named_views, path: str, strict: bool, used: set) -> None:
    """Copy the checkpoint tensors of ``state`` into the fused-layout ``(name, view)`` pairs."""
    with torch.no_grad():
        for name, view in named_views:
            if (name.endswith("mlp.experts.gate_up_proj") or name.endswith("mlp.experts.down_proj")) and name in state:
                src = state[name]
                if src.shape[0] != view.shape[0]:
                    off = _expert_offset(cfg, view)
                    src = src[off : off + view.shape[0]]
                view.copy_(src.to(view.dtype))
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


def save_hf_checkpoint_sharded(sharding, out_dir: str, dtype: Optional[torch.dtype] = None) -> List[str]:
    """HF checkpoint of layer-sharded parameters (``parallel/zero3.py``): every unit is all-gathered
    once (a collective over the ranks) and rank ``u % W`` writes unit ``u`` as its own file, so the
    writes run in parallel with no rank holding more than one unit; rank 0 writes config and index."""
    from safetensors.torch import save_file

    cfg, units, rank, world = sharding.cfg, sharding.units, sharding.rank, sharding.world
    os.makedirs(out_dir, exist_ok=True)
    n = len(units)
    fname = lambda i: f"model-{i + 1:05d}-of-{n:05d}.safetensors"  # noqa: E731
    index = {u.name: i for i, u in enumerate(units)}
    written: List[str] = []

    def write(u, views):
        i = index[u.name]
        if i % world != rank:
            return
        tensors = {}
        for name in u.names:
            for hf, t in hf_items(cfg, name, views[name]):
                tt = t.detach() if dtype is None else t.detach().to(dtype)
                tensors[hf] = tt.to("cpu").contiguous()
        save_file(tensors, os.path.join(out_dir, fname(i)), metadata={"format": "pt"})
        written.append(fname(i))

    sharding.for_each_unit_gathered(write)
    if rank == 0:
        cfg.save(out_dir)
        weight_map, total = {}, 0
        meta = torch.empty(sharding.layout.total_numel, dtype=dtype or sharding.dtype, device="meta")
        for i, u in enumerate(units):
            for name in u.names:
                s = sharding.layout.slots[name]
                for hf, t in hf_items(cfg, name, meta[s.offset : s.offset + s.numel].view(s.shape)):
                    weight_map[hf] = fname(i)
                    total += t.numel() * t.element_size()
        with open(os.path.join(out_dir, "model.safetensors.index.json"), "w", encoding="utf-8") as f:
            json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)
    return written


def load_hf_checkpoint_sharded(sharding, path: str, strict: bool = True) -> None:
    """Fill this rank's shards of layer-sharded parameters from an HF checkpoint (unit by unit; only
    the files of each unit are read)."""
    cfg = sharding.cfg
    used: set = set()

    def fill(u, views):
        meta = torch.empty(sharding.layout.total_numel, dtype=sharding.dtype, device="meta")
        wanted = []
        for name in u.names:
            s = sharding.layout.slots[name]
            wanted += [hf for hf, _ in hf_items(cfg, name, meta[s.offset : s.offset + s.numel].view(s.shape))]
            if ".mlp.experts." in name:
                wanted.append(name)
        state = read_hf_state(path, wanted)
        _load_views(cfg, state, [(name, views[name]) for name in u.names], path, strict, used)

    sharding.for_each_unit_gathered(fill, write_back=True)


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
