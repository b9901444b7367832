"""Rollout workers in their own processes, talking to their engine over a Unix-domain socket.

The reference runs every rollout worker as its own Ray actor process (accerl_agent/agent_textworld.py:
3072-3082), so environment stepping, tokenisation and episode assembly never compete for one
interpreter lock with the inference engine's host-side scheduler. Here the engine process serves
``request_batch`` on a Unix socket (``EngineRequestServer``) and each worker process runs its
``RolloutWorker`` coroutines against an ``EngineClient`` with the same ``request_batch`` surface.
Samples still go straight from the worker process to the trainer's sample queue.

Wire format: 4-byte little-endian length, then a pickled tuple.
  worker -> engine   ("req", id, input ids as int32 bytes, max_tokens)
  engine -> worker   ("res", id, tokens, logprobs, versions, stop_reason) or ("err", id, message)
"""

from __future__ import annotations

import asyncio
import itertools
import os
import pickle
import struct
import traceback
from typing import Any, Dict, List, Optional

import numpy as np

from .generation import InferenceResult

_LEN = struct.Struct("<I")


def _frame(obj) -> bytes:
    body = pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL)
    return _LEN.pack(len(body)) + body


async def _read_frame(reader: asyncio.StreamReader):
    try:
        head = await reader.readexactly(_LEN.size)
        body = await reader.readexactly(_LEN.unpack(head)[0])
    except (asyncio.IncompleteReadError, ConnectionError):
        return None
    return pickle.loads(body)


class EngineRequestServer:
    """Serves ``service.request_batch`` to worker processes; requests run concurrently and answers
    return in completion order (tagged with their request id)."""

    def __init__(self, service, path: str):
        self.service = service
        self.path = path
        self._server = None
        self._tasks: set = set()
        self._writers: set = set()

    async def start(self) -> None:
        if os.path.exists(self.path):
            os.unlink(self.path)
        self._server = await asyncio.start_unix_server(self._connection, path=self.path)

    async def _connection(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter) -> None:
        lock = asyncio.Lock()
        mine: set = set()
        self._writers.add(writer)
        try:
            while True:
                msg = await _read_frame(reader)
                if msg is None:
                    break
                _, rid, ids, max_tokens = msg
                t = asyncio.create_task(self._answer(rid, np.frombuffer(ids, dtype=np.int32).tolist(), max_tokens,
                                                     writer, lock))
                mine.add(t)
                self._tasks.add(t)
                t.add_done_callback(mine.discard)
                t.add_done_callback(self._tasks.discard)
        finally:
            for t in list(mine):
                t.cancel()
            self._writers.discard(writer)
            writer.close()

    async def _answer(self, rid: int, ids: List[int], max_tokens: int, writer, lock) -> None:
        try:
            r = await self.service.request_batch(ids, int(max_tokens))
            out = ("res", rid, r.output_tokens, r.output_logprobs, r.output_versions, r.stop_reason)
        except asyncio.CancelledError:
            raise
        except Exception as exc:
            out = ("err", rid, f"{type(exc).__name__}: {exc}")
        async with lock:
            try:
                writer.write(_frame(out))
                await writer.drain()
            except ConnectionError:
                pass  # the worker process went away; nothing to answer

    async def close(self) -> None:
        for t in list(self._tasks):
            t.cancel()
        for w in list(self._writers):  # established connections keep wait_closed() waiting
            w.close()
        if self._server is not None:
            self._server.close()
            await self._server.wait_closed()
            self._server = None
        if os.path.exists(self.path):
            os.unlink(self.path)


class EngineClient:
    """``request_batch`` of the inference service, forwarded to the engine process."""

    def __init__(self, path: str):
        self.path = path
        self._ids = itertools.count()
        self._pending: Dict[int, asyncio.Future] = {}
        self._reader = None
        self._writer = None
        self._read_task = None

    async def connect(self) -> None:
        self._reader, self._writer = await asyncio.open_unix_connection(self.path)
        self._read_task = asyncio.create_task(self._read_loop())

    async def _read_loop(self) -> None:
        while True:
            msg = await _read_frame(self._reader)
            if msg is None:
                break
            fut = self._pending.pop(msg[1], None)
            if fut is None or fut.done():
                continue
            if msg[0] == "res":
                fut.set_result(InferenceResult(list(msg[2]), list(msg[3]), list(msg[4]), msg[5]))
            else:
                fut.set_exception(RuntimeError(f"engine request failed: {msg[2]}"))
        err = ConnectionError("the engine process closed the request socket")
        for fut in self._pending.values():
            if not fut.done():
                fut.set_exception(err)
        self._pending.clear()

    async def request_batch(self, input_ids: List[int], infer_max_tokens: int) -> InferenceResult:
        rid = next(self._ids)
        fut = asyncio.get_running_loop().create_future()
        self._pending[rid] = fut
        self._writer.write(_frame(("req", rid, np.asarray(input_ids, dtype=np.int32).tobytes(),
                                   int(infer_max_tokens))))
        await self._writer.drain()
        return await fut

    async def close(self) -> None:
        if self._writer is not None:
            self._writer.close()
        if self._read_task is not None:
            self._read_task.cancel()


def worker_process_main(args, path: str, worker_ids: List[int], replay_queues, stats_queue, stop_event,
                        error_queue) -> None:
    """Body of one rollout-worker process: its workers play episodes until ``stop_event`` is set."""
    try:
        asyncio.run(_worker_process(args, path, worker_ids, replay_queues, stats_queue, stop_event))
    except BaseException:
        error_queue.put((tuple(worker_ids), traceback.format_exc()))
        raise


def _make_tokenizer(args):
    if args.env == "textworld":
        from ..trainer.actor import _load_tokenizer

        return _load_tokenizer(args)
    if args.env == "gsm8k":
        from ..core.tokenizer import load_tokenizer
        from ..models.config import resolve_model_config

        return load_tokenizer(args.model_path, args.trust_remote_code,
                              vocab_size=resolve_model_config(args.model_path).vocab_size, fallback=True)
    return None


def make_workers(args, infer, worker_ids: List[int], replay_queues, stats_queue, tokenizer=None) -> List[Any]:
    """The rollout workers of ``worker_ids`` against ``infer`` (an inference service or a client)."""
    world = len(replay_queues)

    def sink_for(wid):
        q = replay_queues[wid % world]
        return lambda samples: q.put(samples)

    def stats_sink(*rec):
        stats_queue.put(rec)

    if args.env == "gsm8k":
        from .math_worker import MathRolloutWorker, load_math_examples

        examples = load_math_examples(args)
        return [MathRolloutWorker(args, infer, wid, sink_for(wid), stats_sink, tokenizer=tokenizer, examples=examples)
                for wid in worker_ids]
    from .worker import RolloutWorker

    return [RolloutWorker(args, infer, wid, sink_for(wid), stats_sink, tokenizer=tokenizer) for wid in worker_ids]


async def _worker_process(args, path, worker_ids, replay_queues, stats_queue, stop_event) -> None:
    client = EngineClient(path)
    await client.connect()
    workers = make_workers(args, client, worker_ids, replay_queues, stats_queue, tokenizer=_make_tokenizer(args))
    tasks = [asyncio.create_task(w.run()) for w in workers]
    try:
        while not stop_event.is_set():
            done = [t for t in tasks if t.done()]
            for t in done:
                if t.exception() is not None:
                    raise t.exception()
            if len(done) == len(tasks):
                return
            await asyncio.sleep(0.1)
        for w in workers:
            await w.stop()
        _, pending = await asyncio.wait(tasks, timeout=float(getattr(args, "rollout_stop_timeout", 10.0)))
        for t in pending:
            t.cancel()
    finally:
        await client.close()


class WorkerProcesses:
    """The worker processes of one engine: ``procs`` processes share the engine's worker ids."""

    def __init__(self, args, service, worker_ids: List[int], replay_queues, stats_queue, procs: int):
        import multiprocessing as mp
        import tempfile

        self.args = args
        self.ctx = mp.get_context("spawn")
        self.dir = tempfile.mkdtemp(prefix="accerl-eng-")
        self.server = EngineRequestServer(service, os.path.join(self.dir, "engine.sock"))
        self.groups = [g for g in (worker_ids[i::procs] for i in range(max(procs, 1))) if g]
        self.replay_queues = replay_queues
        self.stats_queue = stats_queue
        self.stop_event = self.ctx.Event()
        self.errors = self.ctx.Queue()
        self.procs: List[Any] = []

    async def start(self) -> int:
        await self.server.start()
        for g in self.groups:
            p = self.ctx.Process(target=worker_process_main, name=f"rollout-{g[0]}", daemon=True,
                                 args=(self.args, self.server.path, g, self.replay_queues, self.stats_queue,
                                       self.stop_event, self.errors))
            p.start()
            self.procs.append(p)
        return sum(len(g) for g in self.groups)

    def check(self) -> Optional[str]:
        for g, p in zip(self.groups, self.procs):
            if not p.is_alive():
                detail = ""
                try:
                    ids, tb = self.errors.get_nowait()
                    detail = f": {tb.strip().splitlines()[-1]}"
                except Exception:
                    pass
                return f"rollout worker process for workers {g} exited with code {p.exitcode}{detail}"
        return None

    async def stop(self, timeout: float) -> Dict[str, int]:
        self.stop_event.set()
        stopped = killed = 0
        for p in self.procs:
            await asyncio.to_thread(p.join, timeout + 5.0)
            if p.is_alive():
                p.terminate()
                p.join(5.0)
                killed += 1
            else:
                stopped += 1
        await self.server.close()
        return {"stopped": stopped, "cancelled": killed}
