"""The RL train worker: one per GPU (or CPU rank), same public surface as the reference's
``FSDPTrainWorker`` (agent_textworld.py:419-1570):

``train_until_next_sync(n)``, ``get_weight_metadata(scope)``, ``save_checkpoint(dir, tag)``,
``get_replay_stats()``, ``close()``, plus ``flat_weights(scope)`` for the in-place weight sync.

Varlen optimizer step (agent_textworld.py:1153-1297): prepare ``grad_accum_steps`` CPU packs,
all-reduce(MIN) a success flag so one rank's failure fails every rank, all-reduce the global valid
target-token count, then per pack: pinned host->device copy, forward through the response-only LM head,
the fused policy-objective kernel (d loss / d logprob scaled by 1/global_tokens), backward with
weight gradients accumulated in fp32; finally all-reduce the float64 statistics, clip at 1.0 and the
sharded AdamW step with the warm-up + cosine learning rate.

Padded steps (the reference default) run the same varlen kernels on the unpadded rows and apply the
padded objective (per-sample / per-response means, optional advantage normalisation) to the logprobs.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import time
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from .. import ops
from ..utils import nvtx
from ..algo.objectives import ObjectiveConfig, normalize_advantages, padded_loss
from ..algo.packing import (
    make_padded_collate,
    make_varlen_batch,
    padded_to_varlen,
    prepare_rl_sample,
    select_varlen_pack,
    version_lag_stats,
)
from ..algo.schedule import warmup_cosine_lr
from ..core.sample import IGNORE_INDEX, PreparedVarlenPack, RLSample
from ..models.config import resolve_model_config
from ..models.hf_io import load_hf_checkpoint, save_hf_checkpoint, vllm_weight_metadata
from ..models.transformer import build_model
from ..parallel import balance
from ..parallel.fsdp import ShardedAdamW, dist_ready
from ..parallel.expert_parallel import ExpertParallel, expert_partition


def set_seed(seed: int) -> None:
    random.seed(seed)
    np.random.seed(seed % (2**32))
    torch.manual_seed(seed)


def pick_device(name: str) -> torch.device:
    if name == "auto":
        if torch.cuda.is_available():
            return torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)) % torch.cuda.device_count())
        return torch.device("cpu")
    if name == "cuda":
        return torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)) % torch.cuda.device_count())
    return torch.device(name)


def pick_dtype(name: str, device: torch.device) -> torch.dtype:
    if name == "float32":
        return torch.float32
    if name == "float16":
        return torch.float16
    if name == "bfloat16":
        return torch.bfloat16
    return torch.bfloat16 if device.type == "cuda" else torch.float32


@dataclass
class DevicePack:
    batch: Dict[str, torch.Tensor]
    max_seqlen: int
    old_lp: torch.Tensor
    adv: torch.Tensor
    h2d_bytes: int
    # backing buffers: int64 [ids | positions | labels | prediction indices], float32 [old lp | adv],
    # int32 cu_seqlens (what moves when a pack is computed on another rank)
    raw: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None

    @staticmethod
    def from_raw(ints: torch.Tensor, floats: torch.Tensor, cu: torch.Tensor, max_seqlen: int,
                 h2d_bytes: int = 0) -> "DevicePack":
        n = floats.numel() // 2
        T = (ints.numel() - 2 * n) // 2
        batch = {
            "input_ids": ints[:T],
            "position_ids": ints[T : 2 * T],
            "target_labels": ints[2 * T : 2 * T + n],
            "prediction_indices": ints[2 * T + n :],
            "cu_seqlens": cu,
        }
        return DevicePack(batch, max_seqlen, floats[:n], floats[n:], h2d_bytes, (ints, floats, cu))


class PinnedStager:
    """Ring of reusable pinned host buffers for the per-pack host->device copies.

    A slot is handed out again only after the copies issued from it have completed (a CUDA event
    recorded behind them), so the host never overwrites memory an in-flight copy still reads."""

    def __init__(self, device: torch.device, slots: int = 4):
        self.device = device
        self.pin = device.type == "cuda"
        self._slots: List[Dict[str, torch.Tensor]] = [{} for _ in range(slots)]
        self._events: List[Optional[torch.cuda.Event]] = [None] * slots
        self._next = 0
        self._cur = 0

    def acquire(self) -> int:
        i = self._next
        self._next = (self._next + 1) % len(self._slots)
        ev = self._events[i]
        if ev is not None:
            ev.synchronize()
        self._cur = i
        return i

    def buffer(self, name: str, numel: int, dtype: torch.dtype) -> torch.Tensor:
        bufs = self._slots[self._cur]
        b = bufs.get(name)
        if b is None or b.numel() < numel:
            b = torch.empty(max(numel, 1024), dtype=dtype, pin_memory=self.pin)
            bufs[name] = b
        return b[:numel]

    def release(self) -> None:
        """Record completion of the copies just issued from the current slot."""
        if self.pin:
            ev = torch.cuda.Event()
            ev.record()
            self._events[self._cur] = ev


class TrainWorker:
    def __init__(
        self,
        args: argparse.Namespace,
        rank: int = 0,
        fsdp_world_size: int = 1,
        fsdp_master_addr: Optional[str] = None,
        fsdp_master_port: Optional[int] = None,
        replay_buffer=None,
        device: Optional[torch.device] = None,
        tokenizer=None,
    ):
        self.args = args
        self.rank = rank
        self.fsdp_world_size = fsdp_world_size
        self.balance_packs = bool(getattr(args, "balance_packs", True))
        self.last_balance: Dict[str, float] = {}
        self.replay_buffer = replay_buffer
        self.device = device or pick_device(getattr(args, "device", "auto"))
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        if fsdp_world_size > 1 and not dist_ready():
            if fsdp_master_addr:
                os.environ["MASTER_ADDR"] = fsdp_master_addr
            if fsdp_master_port:
                os.environ["MASTER_PORT"] = str(fsdp_master_port)
            backend = "nccl" if self.device.type == "cuda" else "gloo"
            from datetime import timedelta

            dist.init_process_group(backend=backend, rank=rank, world_size=fsdp_world_size,
                                    timeout=timedelta(seconds=int(os.environ.get("ACCERL_PG_TIMEOUT", "600"))))
        set_seed(args.seed + rank)
        self.cfg = resolve_model_config(args.model_path)
        self.dtype = pick_dtype(args.dtype, self.device)
        use_ep = bool(getattr(args, "expert_parallel", False)) and self.cfg.num_experts > 0 and fsdp_world_size > 1
        # expert-partitioned storage: this rank's parameter buffer, gradients and optimizer state hold
        # only its routed experts; the replicated part is laid out first and sharded by the optimizer
        self.expert_partitioned = use_ep and getattr(args, "expert_storage", "partitioned") == "partitioned"
        model_cfg = expert_partition(self.cfg, rank, fsdp_world_size) if self.expert_partitioned else self.cfg
        has_ckpt = os.path.isdir(args.model_path) and any(f.endswith(".safetensors") for f in os.listdir(args.model_path))
        self.sharding = None
        if getattr(args, "shard_params", False):
            # parameters, gradients and optimizer state sharded per layer (parallel/zero3.py)
            if use_ep:
                raise ValueError("--shard-params cannot be combined with --expert-parallel")
            from ..models.hf_io import load_hf_checkpoint_sharded
            from ..parallel.zero3 import LayerShardedParams, ShardedParamAdamW

            self.sharding = LayerShardedParams(self.cfg, self.device, self.dtype, train_mode=args.train_mode)
            self.model = self.sharding.model
            self.model.gradient_checkpointing = bool(args.gradient_checkpointing)
            if has_ckpt:
                load_hf_checkpoint_sharded(self.sharding, args.model_path)
            else:
                self.model.init_weights(seed=args.seed)
            self.optimizer = ShardedParamAdamW(self.sharding, lr=args.learning_rate, weight_decay=args.weight_decay)
        else:
            self.model = build_model(model_cfg, args.train_mode, self.device, self.dtype, pad_to=fsdp_world_size,
                                     experts_last=self.expert_partitioned)
            self.model.gradient_checkpointing = bool(args.gradient_checkpointing)
            if has_ckpt:
                load_hf_checkpoint(self.model, args.model_path)
            else:
                self.model.init_weights(seed=args.seed)
            if self.model.layout.trainable_numel == 0:
                raise RuntimeError(f"No trainable parameters found for mode: {args.train_mode}")
            self.optimizer = ShardedAdamW(self.model, lr=args.learning_rate, weight_decay=args.weight_decay)
        if use_ep:
            if getattr(args, "train_packing", "padded") == "varlen" and args.train_token_budget:
                max_tokens = int(args.train_token_budget)
            else:
                max_tokens = int(args.batch_size) * int(args.max_length)
            self.model.expert_parallel = ExpertParallel(self.cfg, max_tokens=max_tokens, device=self.device,
                                                        dtype=self.dtype)
        self.tokenizer = tokenizer
        self.pad_token_id = self._pad_token_id(tokenizer)
        self.collate_fn = make_padded_collate(self.pad_token_id)
        self.obj_cfg = ObjectiveConfig(
            clip_mode=args.clip_mode,
            clip_eps=args.clip_eps,
            gipo_sigma=args.gipo_sigma,
            sapo_tau_pos=args.sapo_tau_pos,
            sapo_tau_neg=args.sapo_tau_neg,
            kl_coef=args.old_new_kl_coef,
        )
        self.train_micro_step = 0
        self.optimizer_step = 0
        self.pending_prepared_samples: List[RLSample] = []
        self.stager = PinnedStager(self.device)
        self.last_h2d_bytes = 0
        self.last_pack_stats: Dict[str, float] = {}
        if getattr(args, "resume_from", None):
            self.load_checkpoint(args.resume_from)
        if rank == 0:
            total = sum(s.numel for s in self.model.layout.slots.values())
            trainable = sum(s.numel for s in self.model.layout.slots.values() if s.trainable)
            print(f"[train] Parameter count: trainable={trainable:,} / total={total:,} ({trainable / total:.4%})")
            print(f"[rank {rank}] train worker ready on {self.device} ({self.dtype}).")

    # ------------------------------------------------------------------ helpers
    def _pad_token_id(self, tokenizer) -> int:
        if tokenizer is not None:
            if getattr(tokenizer, "pad_token_id", None) is not None:
                return int(tokenizer.pad_token_id)
            if getattr(tokenizer, "eos_token_id", None) is not None:
                return int(tokenizer.eos_token_id)
        return int(self.cfg.eos_token_id)

    def get_rank(self) -> int:
        return self.rank

    def get_replay_stats(self) -> Dict[str, int]:
        return self.replay_buffer.get_stats()

    def current_lr(self) -> float:
        if getattr(self.args, "lr_schedule", "warmup_cosine") == "constant":
            return float(self.args.learning_rate)
        return warmup_cosine_lr(self.optimizer_step, self.args.learning_rate, self.args.lr_warmup_steps,
                                self.args.max_steps)

    def close(self) -> None:
        if dist_ready():
            dist.destroy_process_group()

    def _poll(self, attempt, describe):
        """Call ``attempt()`` until it returns something truthy, sleeping ``--replay-wait-sleep-seconds``
        between calls; after ``--replay-sample-timeout-seconds`` (0: no limit) raise TimeoutError with
        the message ``describe()`` builds."""
        limit = self.args.replay_sample_timeout_seconds
        deadline = time.monotonic() + limit if limit > 0 else None
        while True:
            got = attempt()
            if got:
                return got
            if deadline is not None and time.monotonic() >= deadline:
                raise TimeoutError(describe())
            time.sleep(self.args.replay_wait_sleep_seconds)

    def _wait_for_warmup(self) -> Dict[str, int]:
        need = self.args.min_replay_size_per_rank

        def ready():
            st = self.get_replay_stats()
            return st if st["size"] >= need else None

        def describe():
            st = self.get_replay_stats()
            return (f"Timed out waiting for replay warmup: rank={self.rank} size={st['size']} "
                    f"min_replay_size_per_rank={need} stats={st}")

        return self._poll(ready, describe)

    def _draw_prepared(self, n: int, into: List[RLSample], limit: Optional[int] = None) -> int:
        """Draw ``n`` replay samples, append the ones that survive preparation to ``into`` (at most
        ``limit`` in total); returns how many were drawn."""
        drawn = self.replay_buffer.sample(n)
        for s in drawn:
            prepared = prepare_rl_sample(s, self.args.rl_algorithm, self.args.max_length)
            if prepared is not None and (limit is None or len(into) < limit):
                into.append(prepared)
        return len(drawn)

    def _all_reduce(self, t: torch.Tensor, op=None) -> torch.Tensor:
        if dist_ready() and self.fsdp_world_size > 1:
            dist.all_reduce(t, op=op or dist.ReduceOp.SUM)
        return t

    # ------------------------------------------------------------------ varlen packs
    def _next_varlen_cpu_pack(self, trainer_version: float) -> PreparedVarlenPack:
        t0 = time.perf_counter()
        self._wait_for_warmup()
        pool = self.args.train_pack_candidate_pool_size
        if not self.pending_prepared_samples:
            # candidates carry over between packs; refill only when every candidate was used
            self._poll(lambda: self._draw_prepared(pool, self.pending_prepared_samples) and self.pending_prepared_samples,
                       lambda: f"Timed out waiting for valid replay candidates: rank={self.rank} target={pool} "
                               f"stats={self.get_replay_stats()}")
        selected, remaining = select_varlen_pack(
            self.pending_prepared_samples, self.args.train_token_budget, self.args.batch_size
        )
        if not selected:
            longest = max(len(s.input_ids) for s in self.pending_prepared_samples)
            raise RuntimeError(
                f"No replay sample fits in --train-token-budget: longest_pending={longest} "
                f"budget={self.args.train_token_budget}"
            )
        self.pending_prepared_samples = remaining
        batch = make_varlen_batch(selected)
        valid = int(batch["target_indices"].numel())
        lag_sum, count = version_lag_stats(selected, trainer_version)
        total = int(batch["input_ids"].numel())
        return PreparedVarlenPack(
            batch=batch,
            valid_token_count=valid,
            max_seqlen=max(len(s.input_ids) for s in selected),
            version_lag_sum=lag_sum,
            sample_count=count,
            total_tokens=total,
            pack_cpu_ms=(time.perf_counter() - t0) * 1e3,
        )

    @staticmethod
    def pack_to_device_bytes(pack: PreparedVarlenPack) -> int:
        """Host->device bytes of ``pack_to_device(pack)``."""
        T = int(pack.batch["input_ids"].numel())
        n = int(pack.batch["target_indices"].numel())
        return (2 * T + 2 * n) * 8 + 2 * n * 4 + int(pack.batch["cu_seqlens"].numel()) * 4

    def pack_to_device(self, pack: PreparedVarlenPack) -> DevicePack:
        """Stage a CPU pack in pinned memory and copy it to the device (async on the current stream)."""
        b = pack.batch
        T = b["input_ids"].numel()
        tgt = b["target_indices"]
        n = tgt.numel()
        cu = b["cu_seqlens"]
        if int(cu[-1]) != T or n == 0 or int(b["prediction_indices"].max()) >= T or pack.max_seqlen > T:
            raise RuntimeError(f"inconsistent pack: T={T} cu_last={int(cu[-1])} targets={n}")
        labels = b["labels"].index_select(0, tgt)
        if self.args.rl_algorithm == "grpo":
            adv = b["sample_advantages"].index_select(0, b["sequence_ids"].index_select(0, tgt))
        else:
            adv = b["token_advantages"].index_select(0, tgt)
        old = b["old_logprobs"].index_select(0, tgt)
        self.stager.acquire()
        ints = self.stager.buffer("i64", 2 * T + 2 * n, torch.int64)
        ints[:T].copy_(b["input_ids"].view(-1))
        ints[T : 2 * T].copy_(b["position_ids"].view(-1))
        ints[2 * T : 2 * T + n].copy_(labels)
        ints[2 * T + n :].copy_(b["prediction_indices"])
        floats = self.stager.buffer("f32", 2 * n, torch.float32)
        floats[:n].copy_(old)
        floats[n:].copy_(adv)
        cu_h = self.stager.buffer("i32", b["cu_seqlens"].numel(), torch.int32)
        cu_h.copy_(b["cu_seqlens"])
        if self.device.type == "cuda":
            ints_d = ints.to(self.device, non_blocking=True)
            floats_d = floats.to(self.device, non_blocking=True)
            cu_d = cu_h.to(self.device, non_blocking=True)
        else:  # the staging buffers are reused: CPU packs own copies
            ints_d, floats_d, cu_d = ints.clone(), floats.clone(), cu_h.clone()
        self.stager.release()
        h2d = ints.numel() * 8 + floats.numel() * 4 + cu_h.numel() * 4
        return DevicePack.from_raw(ints_d, floats_d, cu_d, pack.max_seqlen, h2d)

    def _prepare_varlen_optimizer_window(self, trainer_version: float) -> List[PreparedVarlenPack]:
        window = None
        local_error = None
        try:
            window = [self._next_varlen_cpu_pack(trainer_version) for _ in range(self.args.grad_accum_steps)]
        except Exception as exc:  # propagated to every rank below
            local_error = repr(exc)
            print(f"[rank {self.rank}] Varlen window preparation failed: {local_error}")
        if self.fsdp_world_size > 1:
            flag = torch.tensor([0 if local_error else 1], dtype=torch.int32, device=self._comm_device())
            self._all_reduce(flag, dist.ReduceOp.MIN)
            ok = int(flag.item()) == 1
        else:
            ok = local_error is None
        if not ok:
            raise RuntimeError(
                "At least one FSDP rank failed to prepare its Varlen optimizer window; see per-rank logs for the "
                f"original error. local_error={local_error}"
            )
        assert window is not None
        return window

    def _comm_device(self) -> torch.device:
        if dist_ready() and dist.get_backend() == "nccl":
            return self.device
        return torch.device("cpu")

    def run_varlen_step_on_device(self, packs: List[DevicePack], global_tokens: int, timer=None) -> torch.Tensor:
        """Forward/backward of already-staged packs; returns the float64[3] statistics (device).
        ``timer`` (a ``utils.timing.PhaseTimer``) marks forward and backward of every pack."""
        stats = torch.zeros(3, dtype=torch.float64, device=self.device)
        scale = 1.0 / float(global_tokens)
        for dp in packs:
            lp, ctx = self.model.forward_logprobs(dp.batch, dp.max_seqlen)
            dlp, st = ops.policy_loss(lp, dp.old_lp, dp.adv, self.obj_cfg, loss_scale=scale)
            if timer is not None:
                timer.mark("forward")
            self.model.backward_from_logprobs(dlp, ctx)
            stats += st.to(stats.device)
            if timer is not None:
                timer.mark("backward")
            self.train_micro_step += 1
            del ctx, lp, dlp
        return stats

    def _balance_window(self, window: List[PreparedVarlenPack]) -> Tuple[List[Any], int]:
        """Spread the window's packs over the ranks by estimated work (``parallel/balance.py``).
        Returns this rank's work list -- its own CPU packs still to be staged, and packs received from
        other ranks as ``DevicePack`` -- and the global target-token count (every rank's packs)."""
        local_tokens = sum(p.valid_token_count for p in window)
        if self.fsdp_world_size == 1 or not dist_ready():
            return list(window), local_tokens
        meta = np.zeros((len(window), 5), dtype=np.float64)
        for i, p in enumerate(window):
            lens = np.diff(p.batch["cu_seqlens"].numpy().astype(np.int64))
            meta[i] = (balance.pack_cost(self.cfg, lens, p.valid_token_count), p.total_tokens, p.valid_token_count,
                       len(lens), p.max_seqlen)
        meta_all = balance.gather_meta(meta)  # also replaces the global target-token all-reduce
        global_tokens = int(round(meta_all[:, :, 2].sum()))
        if not self.balance_packs:
            return list(window), global_tokens
        assign, moves = balance.plan(meta_all)
        outgoing = {mv.index: self.pack_to_device(window[mv.index]).raw for mv in moves if mv.src == self.rank}
        received = balance.exchange(moves, self.rank, outgoing, self.device)
        max_len = {(mv.src, mv.index): mv.max_seqlen for mv in moves}
        work: List[Any] = []
        for owner, i in assign[self.rank]:
            if owner == self.rank:
                work.append(window[i])
            else:
                work.append(DevicePack.from_raw(*received[(owner, i)], max_len[(owner, i)]))
        self.last_balance = {"moved_in": sum(1 for o, _ in assign[self.rank] if o != self.rank),
                             "rank_cost": float(sum(meta_all[o, i, 0] for o, i in assign[self.rank])),
                             "mean_cost": float(meta_all[:, :, 0].sum() / self.fsdp_world_size)}
        return work, global_tokens

    def stage_window(self, trainer_version: float = 0.0) -> Tuple[List[DevicePack], int]:
        """Prepare one optimizer window (balanced over the ranks) and leave its packs resident on the
        device (benchmarks)."""
        window = self._prepare_varlen_optimizer_window(trainer_version)
        work, global_tokens = self._balance_window(window)
        packs = []
        for item in work:
            dp = item if isinstance(item, DevicePack) else self.pack_to_device(item)
            packs.append(DevicePack.from_raw(*(t.clone() for t in dp.raw), dp.max_seqlen, dp.h2d_bytes))
        return packs, global_tokens

    def train_step_on_device(self, packs: List[DevicePack], global_tokens: int, timer=None) -> torch.Tensor:
        """One optimizer step over device-resident packs: forward/backward of every pack, the
        statistics all-reduce and the sharded AdamW step (no host<->device traffic). ``timer``
        (a ``utils.timing.PhaseTimer``, first mark already taken) splits the step into phases."""
        stats = self.run_varlen_step_on_device(packs, global_tokens, timer)
        if self.fsdp_world_size > 1:
            self._all_reduce(stats)
            if timer is not None:
                timer.mark("stats_allreduce")
        self.optimizer.step(self.current_lr(), timer=timer)
        self.optimizer_step += 1
        return stats

    def _run_varlen_optimizer_step(self, trainer_version: float) -> Dict[str, float]:
        with nvtx.range("train/prepare_window"):
            window = self._prepare_varlen_optimizer_window(trainer_version)
        with nvtx.range("train/balance"):
            work, global_tokens = self._balance_window(window)
        if global_tokens <= 0:
            raise RuntimeError("Global Varlen optimizer window contains no valid response tokens.")
        stats = torch.zeros(3, dtype=torch.float64, device=self.device)
        h2d = sum(self.pack_to_device_bytes(p) for p in window if not any(p is w for w in work))
        scale = 1.0 / float(global_tokens)
        for pack in work:
            with nvtx.range("train/h2d"):
                dp = pack if isinstance(pack, DevicePack) else self.pack_to_device(pack)
            h2d += dp.h2d_bytes
            with nvtx.range("train/forward"):
                lp, ctx = self.model.forward_logprobs(dp.batch, dp.max_seqlen)
            with nvtx.range("train/loss"):
                dlp, st = ops.policy_loss(lp, dp.old_lp, dp.adv, self.obj_cfg, loss_scale=scale)
            with nvtx.range("train/backward"):
                self.model.backward_from_logprobs(dlp, ctx)
            stats += st.to(stats.device)
            self.train_micro_step += 1
            del ctx, lp, dlp, dp
        self.last_h2d_bytes = h2d
        version = torch.tensor([sum(p.version_lag_sum for p in window), sum(p.sample_count for p in window)],
                               dtype=torch.float64, device=self._comm_device())
        if self.fsdp_world_size > 1:
            with nvtx.range("train/stats_allreduce"):
                st_comm = stats.to(self._comm_device())
                self._all_reduce(st_comm)
                stats = st_comm
                self._all_reduce(version)
        lr = self.current_lr()
        with nvtx.range("train/optimizer"):
            self.optimizer.step(lr)
        self.optimizer_step += 1
        policy_sum, kl_sum, clip_count = stats.tolist()
        lag_sum, sample_count = version.tolist()
        self.last_pack_stats = {
            "pack_token_utilization": float(np.mean([p.total_tokens / self.args.train_token_budget for p in window])),
            "pack_sample_count": float(np.mean([p.sample_count for p in window])),
            "pack_max_sequence_length": float(max(p.max_seqlen for p in window)),
            "pack_cpu_ms": float(np.mean([p.pack_cpu_ms for p in window])),
            "total_tokens": float(sum(p.total_tokens for p in window)),
        }
        n = float(global_tokens)
        return {
            "global_policy_sum": policy_sum,
            "global_kl_sum": kl_sum,
            "global_clip_count": clip_count,
            "global_valid_token_count": n,
            "global_version_lag_sum": lag_sum,
            "global_sample_count": sample_count,
            "loss_mean": policy_sum / n + self.args.old_new_kl_coef * kl_sum / n,
            "kl_token_mean": kl_sum / n,
            "clip_fraction": clip_count / n,
            "current_lr": lr,
        }

    # ------------------------------------------------------------------ padded path
    def _next_padded_batch(self, trainer_version: float) -> Tuple[List[RLSample], float]:
        self._wait_for_warmup()
        bs = self.args.batch_size
        collected: List[RLSample] = []
        while len(collected) < bs:  # each draw may lose samples to preparation; draw again for the rest
            self._poll(lambda: self._draw_prepared(bs - len(collected), collected, limit=bs),
                       lambda: f"Timed out waiting for replay samples: rank={self.rank} have={len(collected)} "
                               f"need={bs} stats={self.get_replay_stats()}")
        samples = collected[:bs]
        lag_sum, count = version_lag_stats(samples, trainer_version)
        return samples, lag_sum / count

    def _padded_micro_step(self, samples: List[RLSample]) -> Tuple[float, Dict[str, float], float]:
        batch = self.collate_fn(samples)
        labels = batch["labels"][:, 1:]
        mask = labels.ne(IGNORE_INDEX)
        counts = mask.sum(-1).clamp_min(1)
        valid_pos = mask.nonzero(as_tuple=False)
        if valid_pos.numel() == 0:
            raise RuntimeError("No valid response tokens found for RL loss.")
        sample_idx = valid_pos[:, 0]
        vb = padded_to_varlen(batch)
        L = batch["input_ids"].shape[1]
        # prediction position (row, col) predicts the label at (row, col+1); map to packed rows
        flat_pred = valid_pos[:, 0] * L + valid_pos[:, 1]
        lookup = torch.full((batch["input_ids"].numel(),), -1, dtype=torch.long)
        lookup[vb["flat_index"]] = torch.arange(vb["flat_index"].numel())
        pred_idx = lookup[flat_pred]
        tgt_labels = labels[mask]
        dev = self.device
        dbatch = {
            "input_ids": vb["input_ids"].reshape(-1).to(dev),
            "position_ids": vb["position_ids"].reshape(-1).to(dev),
            "cu_seqlens": vb["cu_seqlens"].to(dev),
            "prediction_indices": pred_idx.to(dev),
            "target_labels": tgt_labels.to(dev),
        }
        lp, ctx = self.model.forward_logprobs(dbatch, vb["max_seqlen"])
        old = batch["old_logprobs"][:, 1:][mask].to(dev)
        if self.args.rl_algorithm == "ppo":
            adv = batch["token_advantages"][:, 1:][mask].to(dev).float()
            if self.args.ppo_normalize_advantages:
                adv = normalize_advantages(adv, self.args.ppo_adv_norm_eps)
            resp_idx = batch["response_indices"][:, 1:][mask].to(dev)
        else:
            adv = batch["sample_advantages"][sample_idx].to(dev).float()
            resp_idx = torch.zeros_like(sample_idx).to(dev)
        x = lp.detach().float().requires_grad_(True)
        with torch.enable_grad():
            loss, stats = padded_loss(x, old, adv, sample_idx.to(dev), resp_idx, counts.to(dev), len(samples),
                                      self.args.rl_algorithm, self.obj_cfg)
            scale = 1.0 / (self.args.grad_accum_steps * max(self.fsdp_world_size, 1))
            (dlp,) = torch.autograd.grad(loss * scale, x)
        self.model.backward_from_logprobs(dlp, ctx)
        return float(loss.item()), stats, float(counts.sum().item())

    # ------------------------------------------------------------------ segments
    def train_until_next_sync(self, num_optimizer_steps: int = 100) -> Dict[str, Any]:
        if num_optimizer_steps < 1:
            raise ValueError("num_optimizer_steps must be >= 1")
        start = self.optimizer_step
        target = min(self.optimizer_step + num_optimizer_steps, self.args.max_steps)
        losses: List[float] = []
        kls: List[float] = []
        clips: List[float] = []
        lags: List[float] = []
        valid_tokens = 0.0
        varlen_steps: List[Dict[str, float]] = []
        while self.optimizer_step < target:
            trainer_version = self.optimizer_step / self.args.sync_every_optimizer_steps
            if self.args.train_packing == "varlen":
                st = self._run_varlen_optimizer_step(trainer_version)
                varlen_steps.append(st)
                if self.rank == 0 and self.optimizer_step % self.args.log_every == 0:
                    print(
                        f"[train] optimizer_step={self.optimizer_step} loss={st['loss_mean']:.6f} "
                        f"kl_token_mean={st['kl_token_mean']:.6f} clip_frac={st['clip_fraction']:.4f} "
                        f"tokens={st['global_valid_token_count']:.0f} lr={st['current_lr']:.8g}"
                    )
                continue
            samples, lag = self._next_padded_batch(trainer_version)
            raw_loss, stats, ntok = self._padded_micro_step(samples)
            losses.append(raw_loss)
            kls.append(stats.get("old_new_kl_k3_token_mean", 0.0))
            clips.append(stats.get("ppo_clip_frac", 0.0))
            lags.append(lag)
            valid_tokens += ntok
            self.train_micro_step += 1
            if self.train_micro_step % self.args.grad_accum_steps != 0:
                continue
            lr = self.current_lr()
            self.optimizer.step(lr)
            self.optimizer_step += 1
            if self.rank == 0 and self.optimizer_step % self.args.log_every == 0:
                print(f"[train] optimizer_step={self.optimizer_step} loss={raw_loss:.6f} "
                      f"kl_token_mean={kls[-1]:.6f} clip_frac={clips[-1]:.4f} lr={lr:.8g}")
        if varlen_steps:
            valid_tokens = sum(s["global_valid_token_count"] for s in varlen_steps)
            psum = sum(s["global_policy_sum"] for s in varlen_steps)
            ksum = sum(s["global_kl_sum"] for s in varlen_steps)
            csum = sum(s["global_clip_count"] for s in varlen_steps)
            kls = [ksum / valid_tokens]
            losses = [(psum + self.args.old_new_kl_coef * ksum) / valid_tokens]
            clips = [csum / valid_tokens]
            lags = [sum(s["global_version_lag_sum"] for s in varlen_steps) /
                    max(sum(s["global_sample_count"] for s in varlen_steps), 1.0)]
        if dist_ready() and self.fsdp_world_size > 1:
            dist.barrier()
        run = self.optimizer_step - start
        summary = {
            "rank": self.rank,
            "optimizer_steps_run": run,
            "optimizer_step": self.optimizer_step,
            "micro_step": self.train_micro_step,
            "reached_max_steps": self.optimizer_step >= self.args.max_steps,
            "segment_loss_mean": sum(losses) / len(losses) if losses else 0.0,
            "segment_kl_mean": sum(kls) / len(kls) if kls else 0.0,
            "segment_clip_frac": sum(clips) / len(clips) if clips else 0.0,
            "segment_valid_tokens": valid_tokens,
            "segment_version_lag_mean": sum(lags) / len(lags) if lags else 0.0,
            "learning_rate": self.optimizer.lr,
        }
        summary.update({f"pack_{k}" if not k.startswith("pack_") else k: v for k, v in self.last_pack_stats.items()})
        return summary

    # ------------------------------------------------------------------ weights / checkpoints
    def get_weight_metadata(self, scope: str = "all"):
        if scope not in ("all", "trainable"):
            raise ValueError(f"Unsupported weight scope: {scope!r}")
        model = self.model
        if self.sharding is not None:  # names and shapes only: a model over meta storage
            model = build_model(self.cfg, "full", torch.device("meta"), self.dtype, with_grads=False)
        return vllm_weight_metadata(model, trainable_only=scope == "trainable")

    def flat_weights(self, scope: str = "all") -> torch.Tensor:
        """The full bf16 compute copy in fused layout. Trainable parameters form a contiguous prefix,
        so a trainable-scope sync is a single contiguous range."""
        if self.sharding is not None:  # this rank's shards of every unit (the engine maps every rank)
            if scope == "trainable":
                return self.sharding.local[: self.sharding.n_trainable]
            if scope == "all":
                return self.sharding.local
            raise ValueError(f"Unsupported weight scope: {scope!r}")
        if scope == "trainable":
            return self.model.params[: self.model.layout.trainable_numel]
        if scope == "all":
            return self.model.params
        raise ValueError(f"Unsupported weight scope: {scope!r}")

    def save_checkpoint(self, checkpoint_dir: str, tag: str, save_optimizer: Optional[bool] = None) -> Dict[str, Any]:
        """HF-format weights (as ``agent_textworld.py:1502`` of the reference saves them) plus, with
        ``save_optimizer`` (default ``--save-optimizer-state``), this rank's fp32 master / Adam moment
        shards and the step counters, so ``--resume-from`` continues the same optimisation."""
        if save_optimizer is None:
            save_optimizer = bool(getattr(self.args, "save_optimizer_state", False))
        if not checkpoint_dir:
            raise ValueError("checkpoint_dir must be non-empty")
        if not tag:
            raise ValueError("tag must be non-empty")
        out = os.path.join(checkpoint_dir, tag)
        if dist_ready() and self.fsdp_world_size > 1:
            dist.barrier()
        if self.rank == 0:
            os.makedirs(out, exist_ok=True)
            print(f"[checkpoint] Saving HuggingFace checkpoint to {out} (optimizer_step={self.optimizer_step})")
        if dist_ready() and self.fsdp_world_size > 1:
            dist.barrier()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        if self.sharding is not None:
            from ..models.hf_io import save_hf_checkpoint_sharded

            save_hf_checkpoint_sharded(self.sharding, out)
        else:
            save_hf_checkpoint(self.model, out, rank=self.rank, world=self.fsdp_world_size)
        if save_optimizer:
            torch.save({k: (v.cpu() if torch.is_tensor(v) else v) for k, v in self.optimizer.state_dict().items()},
                       os.path.join(out, f"optimizer_rank{self.rank:05d}.pt"))
        result = {"rank": self.rank, "checkpoint_dir": out, "optimizer_step": self.optimizer_step, "saved": True}
        if self.rank == 0:
            if self.tokenizer is not None and hasattr(self.tokenizer, "save_pretrained"):
                self.tokenizer.save_pretrained(out)
            state = {
                "optimizer_step": self.optimizer_step,
                "train_micro_step": self.train_micro_step,
                "fsdp_world_size": self.fsdp_world_size,
                "train_mode": self.args.train_mode,
                "rl_algorithm": self.args.rl_algorithm,
                "max_steps": self.args.max_steps,
                "sync_every_optimizer_steps": self.args.sync_every_optimizer_steps,
            }
            with open(os.path.join(out, "trainer_state.json"), "w", encoding="utf-8") as f:
                json.dump(state, f, ensure_ascii=False, indent=2, sort_keys=True)
                f.write("\n")
            print(f"[checkpoint] Saved checkpoint to {out}")
        if dist_ready() and self.fsdp_world_size > 1:
            dist.barrier()
        return result

    def load_checkpoint(self, path: str) -> None:
        """Resume: weights from the HF files, optimizer shards and counters when present."""
        if self.sharding is not None:
            from ..models.hf_io import load_hf_checkpoint_sharded

            load_hf_checkpoint_sharded(self.sharding, path)
        else:
            load_hf_checkpoint(self.model, path)
        self.optimizer.refresh_master_from_params()
        opt = os.path.join(path, f"optimizer_rank{self.rank:05d}.pt")
        if os.path.exists(opt):
            state = torch.load(opt, map_location=self.device)
            self.optimizer.load_state_dict(state)
        state_path = os.path.join(path, "trainer_state.json")
        if os.path.exists(state_path):
            with open(state_path, encoding="utf-8") as f:
                st = json.load(f)
            self.optimizer_step = int(st.get("optimizer_step", 0))
            self.train_micro_step = int(st.get("train_micro_step", 0))
