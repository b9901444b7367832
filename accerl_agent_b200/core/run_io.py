"""Run directory artefacts and metric sinks.

* ``save_run_config`` writes ``args.json`` and a copy-pasteable ``command.txt``
  (agent_textworld.py:2864-2905);
* ``checkpoint_tag`` gives ``step-XXXXXX[-suffix]`` (agent_textworld.py:2908-2912);
* ``MetricsWriter`` logs scalars to TensorBoard (same tag names as the reference) and, always, to a
  ``metrics.jsonl`` file in the run directory.
"""

from __future__ import annotations

import json
import os
import shlex
import sys
import time
from typing import Dict, List, Optional


def format_shell_command(argv: List[str]) -> str:
    if not argv:
        return "python"
    command = f"python {shlex.quote(argv[0])}"
    if len(argv) == 1:
        return command
    parts: List[List[str]] = []
    i = 1
    while i < len(argv):
        part = argv[i]
        if part.startswith("-") and i + 1 < len(argv) and not argv[i + 1].startswith("-"):
            parts.append([part, argv[i + 1]])
            i += 2
        else:
            parts.append([part])
            i += 1
    lines = [f"{command} \\"]
    for j, group in enumerate(parts):
        line = "  " + " ".join(shlex.quote(p) for p in group)
        if j + 1 < len(parts):
            line += " \\"
        lines.append(line)
    return "\n".join(lines)


def save_run_config(args, argv: Optional[List[str]] = None) -> None:
    os.makedirs(args.log_dir, exist_ok=True)
    with open(os.path.join(args.log_dir, "args.json"), "w", encoding="utf-8") as f:
        json.dump(vars(args), f, ensure_ascii=False, indent=2, sort_keys=True, default=str)
        f.write("\n")
    with open(os.path.join(args.log_dir, "command.txt"), "w", encoding="utf-8") as f:
        f.write(format_shell_command(sys.argv if argv is None else argv))
        f.write("\n")


def checkpoint_tag(optimizer_step: int, suffix: Optional[str] = None) -> str:
    tag = f"step-{optimizer_step:06d}"
    return f"{tag}-{suffix}" if suffix else tag


class MetricsWriter:
    def __init__(self, log_dir: str):
        os.makedirs(log_dir, exist_ok=True)
        self.log_dir = log_dir
        self._jsonl = open(os.path.join(log_dir, "metrics.jsonl"), "a", encoding="utf-8")
        try:
            from torch.utils.tensorboard import SummaryWriter

            self._tb = SummaryWriter(log_dir)
        except Exception:  # pragma: no cover - tensorboard is optional
            self._tb = None

    def add_scalars(self, scalars: Dict[str, float], step: int) -> None:
        rec = {"step": step, "time": time.time()}
        for tag, value in scalars.items():
            if value is None:
                continue
            rec[tag] = float(value)
            if self._tb is not None:
                self._tb.add_scalar(tag, float(value), step)
        self._jsonl.write(json.dumps(rec) + "\n")

    def flush(self) -> None:
        self._jsonl.flush()
        if self._tb is not None:
            self._tb.flush()

    def close(self) -> None:
        self.flush()
        self._jsonl.close()
        if self._tb is not None:
            self._tb.close()
