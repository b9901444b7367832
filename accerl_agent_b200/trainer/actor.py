"""Trainer process actor: one ``TrainWorker`` per GPU plus its replay shard.

Rollout workers push lists of ``RLSample`` into this rank's sample queue; a background thread moves
them into the local ``ReplayBuffer`` (the reference keeps one replay actor per FSDP rank and each
trainer reads only its own shard, agent_textworld.py:2983-3008).
"""

from __future__ import annotations

import os
import threading
from typing import Any, Dict, Optional

import torch


def _load_tokenizer(args):
    if not os.path.isdir(args.model_path):
        return None
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(args.model_path, local_files_only=True,
                                            trust_remote_code=args.trust_remote_code)
        if tok.pad_token is None:
            tok.pad_token = tok.eos_token
        return tok
    except Exception:
        return None


class TrainerActor:
    def __init__(self, args, rank: int, world: int, master_addr: str, master_port: int, sample_queue,
                 device_index: Optional[int]):
        from ..replay import ReplayBuffer
        from .worker import TrainWorker

        self.rank = rank
        if device_index is not None and torch.cuda.is_available():
            device = torch.device("cuda", device_index)
            torch.cuda.set_device(device)
        else:
            device = torch.device("cpu")
        self.replay = ReplayBuffer(args.replay_capacity, seed=args.seed + rank)
        self.worker = TrainWorker(args, rank, world, master_addr, master_port, replay_buffer=self.replay,
                                  device=device, tokenizer=_load_tokenizer(args))
        if device.type == "cpu":
            self.worker.flat_weights("all").share_memory_()
        self._queue = sample_queue
        self._stop = False
        self._drain = threading.Thread(target=self._drain_samples, daemon=True)
        self._drain.start()

    def _drain_samples(self):
        while not self._stop:
            try:
                samples = self._queue.get(timeout=0.5)
            except Exception:
                continue
            if samples is None:
                break
            self.replay.add_samples(samples)

    def get_rank(self) -> int:
        return self.rank

    def train_until_next_sync(self, n: int) -> Dict[str, Any]:
        return self.worker.train_until_next_sync(n)

    def get_replay_stats(self) -> Dict[str, int]:
        return self.replay.get_stats()

    def get_weight_metadata(self, scope: str = "all"):
        return self.worker.get_weight_metadata(scope)

    def weight_numel(self, scope: str = "all") -> int:
        if self.worker.sharding is not None:
            sh = self.worker.sharding
            if scope == "trainable":
                return int(sum(s.numel for s in sh.layout.slots.values() if s.trainable))
            return int(sh.full_numel())
        return int(self.worker.flat_weights(scope).numel())

    def export_weights_handle(self):
        """Handle that lets another process map this rank's flat bf16 parameters (a CUDA IPC handle of
        the allocation plus the buffer's offset on GPU, a shared-memory handle on CPU). Every rank
        holds the full compute copy after each optimizer step, except for routed experts under
        expert-partitioned storage (the handle then says which rank of how many it is)."""
        from torch.multiprocessing.reductions import reduce_tensor

        params = self.worker.flat_weights("all")
        mcfg = self.worker.model.cfg
        part = {}
        if self.worker.sharding is not None:
            # layer-sharded trainers: this buffer holds this rank's shard of every unit
            part = {"zero3": True, "trainer_rank": self.worker.rank, "world": self.worker.fsdp_world_size,
                    "train_mode": self.worker.args.train_mode}
        elif mcfg.local_experts is not None and mcfg.local_experts != mcfg.num_experts:
            # expert-partitioned storage: the engine needs every rank's buffer and where its experts sit
            part = {"partition": True, "trainer_rank": self.worker.rank, "world": self.worker.fsdp_world_size}
        if params.is_cuda:
            from ..ops._ext import native

            torch.cuda.synchronize(params.device)
            rc, handle, offset = native().ipc_export(params)
            if rc != 0:
                raise RuntimeError(f"cudaIpcGetMemHandle failed with code {rc}")
            probe = bytes(params[:8].view(torch.uint8).cpu().numpy().tobytes())
            return {"kind": "cuda-ipc", "handle": bytes(handle), "offset": int(offset), "numel": params.numel(),
                    "device": params.device.index, "probe": probe, **part}
        return {"kind": "torch", "reduce": reduce_tensor(params), "numel": params.numel(), **part}

    def synchronize(self) -> None:
        if self.worker.device.type == "cuda":
            torch.cuda.synchronize(self.worker.device)

    def save_checkpoint(self, checkpoint_dir: str, tag: str) -> Dict[str, Any]:
        return self.worker.save_checkpoint(checkpoint_dir, tag)

    def close(self) -> None:
        self._stop = True
        self.worker.close()
