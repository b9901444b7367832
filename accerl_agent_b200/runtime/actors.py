"""Process actors: the Ray-free runtime of the async RL loop.

``spawn_actor(factory, *args, env=..., name=...)`` starts a spawned process that builds one object and
serves method calls on it. ``handle.method.remote(*a)`` returns a ``concurrent.futures.Future``;
``handle.method(*a)`` blocks; ``get(futures)`` / ``wait(futures, timeout)`` mirror ``ray.get`` /
``ray.wait``. Coroutine methods run concurrently on the actor's event loop (so ``stop()`` can
interleave with a running ``run()``, as Ray's ``max_concurrency=2`` allows in the reference,
agent_textworld.py:3020-3023); plain methods run one at a time in a worker thread, keeping the loop
responsive. Exceptions travel back with their traceback and are raised by ``get``. A dead actor
process fails every pending call (failure detection for the driver), and ``kill()`` terminates it.
"""

from __future__ import annotations

import asyncio
import concurrent.futures as cf
import importlib
import itertools
import multiprocessing as mp
import os
import pickle
import sys
import threading
import traceback
from typing import Any, Callable, Dict, Iterable, List, Optional, Sequence, Tuple


class ActorError(RuntimeError):
    """An exception raised inside an actor, re-raised in the caller with the remote traceback."""


class ActorDied(RuntimeError):
    pass


def _resolve(factory):
    if isinstance(factory, str):
        mod, _, attr = factory.rpartition(":")
        return getattr(importlib.import_module(mod), attr)
    return factory


def _current_cuda_device() -> Optional[int]:
    torch = sys.modules.get("torch")
    if torch is None or not torch.cuda.is_initialized():
        return None
    return torch.cuda.current_device()


def _select_cuda_device(device: Optional[int]) -> None:
    if device is not None:
        import torch

        torch.cuda.set_device(device)


def _actor_main(factory, args, kwargs, conn, env: Dict[str, str]):
    os.environ.update(env or {})
    obj = None
    send_lock = threading.Lock()

    def send(msg):
        data = pickle.dumps(msg, protocol=pickle.HIGHEST_PROTOCOL)
        with send_lock:
            conn.send_bytes(data)

    try:
        obj = _resolve(factory)(*args, **kwargs)
        send(("ready", None, None))
    except BaseException as exc:  # construction failure
        send(("init_error", None, (repr(exc), traceback.format_exc())))
        return

    loop = asyncio.new_event_loop()
    asyncio.set_event_loop(loop)
    # Plain methods run on a pool thread. The CUDA current device is per thread, so that thread takes
    # the device the constructor selected (an actor drives one GPU); otherwise kernels launched from it
    # would go to device 0.
    device = _current_cuda_device()
    sync_pool = cf.ThreadPoolExecutor(max_workers=1, thread_name_prefix="actor-sync",
                                      initializer=_select_cuda_device, initargs=(device,))
    stopping = asyncio.Event()

    async def handle(call_id, method, a, k):
        try:
            fn = getattr(obj, method)
            if asyncio.iscoroutinefunction(fn):
                res = await fn(*a, **k)
            else:
                res = await loop.run_in_executor(sync_pool, lambda: fn(*a, **k))
                if asyncio.iscoroutine(res):
                    res = await res
            send(("result", call_id, res))
        except BaseException as exc:  # noqa: BLE001 - forwarded to the caller
            try:
                send(("error", call_id, (repr(exc), traceback.format_exc())))
            except Exception:
                pass

    def reader():
        while True:
            try:
                data = conn.recv_bytes()
            except (EOFError, OSError):
                loop.call_soon_threadsafe(stopping.set)
                return
            msg = pickle.loads(data)
            if msg[0] == "call":
                _, call_id, method, a, k = msg
                asyncio.run_coroutine_threadsafe(handle(call_id, method, a, k), loop)
            elif msg[0] == "exit":
                loop.call_soon_threadsafe(stopping.set)
                return

    threading.Thread(target=reader, daemon=True).start()
    loop.run_until_complete(stopping.wait())
    sync_pool.shutdown(wait=False, cancel_futures=True)
    os._exit(0)


class _Method:
    def __init__(self, handle: "ActorHandle", name: str):
        self._h = handle
        self._name = name

    def remote(self, *a, **k) -> cf.Future:
        return self._h._call(self._name, a, k)

    def __call__(self, *a, **k):
        return self._h._call(self._name, a, k).result()


class ActorHandle:
    def __init__(self, proc: mp.Process, conn, name: str):
        self._proc = proc
        self._conn = conn
        self.name = name
        self._pending: Dict[int, cf.Future] = {}
        self._ids = itertools.count()
        self._lock = threading.Lock()
        self._dead: Optional[str] = None
        self._ready = cf.Future()
        self._reader = threading.Thread(target=self._read, daemon=True, name=f"actor-{name}-reader")
        self._reader.start()

    def _read(self):
        while True:
            try:
                data = self._conn.recv_bytes()
            except (EOFError, OSError):
                self._fail_all(f"actor {self.name} (pid {self._proc.pid}) exited")
                return
            kind, call_id, payload = pickle.loads(data)
            if kind == "ready":
                self._ready.set_result(True)
                continue
            if kind == "init_error":
                self._ready.set_exception(ActorError(f"{self.name} failed to start: {payload[0]}\n{payload[1]}"))
                continue
            with self._lock:
                fut = self._pending.pop(call_id, None)
            if fut is None:
                continue
            if kind == "result":
                fut.set_result(payload)
            else:
                fut.set_exception(ActorError(f"{self.name}: {payload[0]}\n--- remote traceback ---\n{payload[1]}"))

    def _fail_all(self, why: str):
        with self._lock:
            self._dead = why
            pending = list(self._pending.values())
            self._pending.clear()
        if not self._ready.done():
            self._ready.set_exception(ActorDied(why))
        for f in pending:
            if not f.done():
                f.set_exception(ActorDied(why))

    def wait_ready(self, timeout: Optional[float] = None) -> None:
        self._ready.result(timeout=timeout)

    def _call(self, method: str, a, k) -> cf.Future:
        fut: cf.Future = cf.Future()
        with self._lock:
            if self._dead:
                fut.set_exception(ActorDied(self._dead))
                return fut
            call_id = next(self._ids)
            self._pending[call_id] = fut
        try:
            self._conn.send_bytes(pickle.dumps(("call", call_id, method, a, k), protocol=pickle.HIGHEST_PROTOCOL))
        except (OSError, BrokenPipeError) as exc:
            self._fail_all(f"actor {self.name} unreachable: {exc!r}")
        return fut

    def __getattr__(self, name: str) -> _Method:
        if name.startswith("_"):
            raise AttributeError(name)
        return _Method(self, name)

    def method(self, name: str) -> _Method:
        """Explicit access to a remote method (also for names that the handle itself defines)."""
        return _Method(self, name)

    @property
    def alive(self) -> bool:
        return self._proc.is_alive() and self._dead is None

    @property
    def pid(self) -> Optional[int]:
        return self._proc.pid

    def stop_process(self, timeout: float = 10.0) -> None:
        """Ask the actor process to exit; kill it if it does not within ``timeout``."""
        try:
            self._conn.send_bytes(pickle.dumps(("exit", None, None, None, None)))
        except Exception:
            pass
        self._proc.join(timeout)
        if self._proc.is_alive():
            self.kill()

    def kill(self) -> None:
        if self._proc.is_alive():
            self._proc.kill()
            self._proc.join(5)


def spawn_actor(factory: Any, *args, env: Optional[Dict[str, str]] = None, name: str = "actor",
                ready_timeout: Optional[float] = 600.0, **kwargs) -> ActorHandle:
    """Start ``factory(*args, **kwargs)`` in a spawned process. ``factory`` may be a class, a
    module-level function, or an ``"module:attr"`` string."""
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe(duplex=True)
    proc = ctx.Process(target=_actor_main, args=(factory, args, kwargs, child, env or {}), name=name, daemon=False)
    proc.start()
    child.close()
    h = ActorHandle(proc, parent, name)
    if ready_timeout is not None:
        h.wait_ready(ready_timeout)
    return h


def get(futures, timeout: Optional[float] = None):
    if isinstance(futures, cf.Future):
        return futures.result(timeout=timeout)
    return [f.result(timeout=timeout) for f in futures]


def wait(futures: Sequence[cf.Future], num_returns: int = 1, timeout: Optional[float] = None):
    done, pending = cf.wait(list(futures), timeout=timeout, return_when=cf.FIRST_COMPLETED)
    ready = [f for f in futures if f in done][:num_returns]
    rest = [f for f in futures if f not in ready]
    return ready, rest
