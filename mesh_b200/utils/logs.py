"""Agent logging: a daily-rotating file log plus console output (``agent/src/observability/
logging.rs:18-74``).

``init_production_logging`` writes ``$MESHNET_HOME/logs/agent.log`` (rotated at midnight, a week
kept, no colour, with logger name and line number) and a short console format; ``MESH_LOG``
overrides the level (``debug``, ``info``, ``warning`` … or per-logger ``mesh.worker=debug,info``).
``init_simple_logging`` is the console-only form for one-shot CLI commands. Both are idempotent:
a second call replaces the handlers the first one installed.
"""
from __future__ import annotations

import logging
import logging.handlers
import os
import sys
from pathlib import Path
from typing import Optional

_INSTALLED = []
FILE_FORMAT = "%(asctime)s %(levelname)s %(name)s:%(lineno)d %(message)s"
CONSOLE_FORMAT = "%(asctime)s %(levelname)s %(message)s"


def _meshnet_home() -> Path:
    h = os.environ.get("MESHNET_HOME")
    return Path(h) if h else Path.home() / ".meshnet"


def _apply_levels(spec: str, default: str) -> int:
    """``spec`` is ``level`` or ``name=level,...,level``; returns the root level."""
    root = logging.getLevelName(default.upper())
    for part in filter(None, (p.strip() for p in spec.split(","))):
        if "=" in part:
            name, lvl = part.split("=", 1)
            logging.getLogger(name.strip()).setLevel(lvl.strip().upper())
        else:
            root = logging.getLevelName(part.upper())
    if not isinstance(root, int):
        raise ValueError(f"unknown log level in {spec!r}")
    return root


def _install(handlers, level: str) -> logging.Logger:
    root = logging.getLogger()
    for h in _INSTALLED:
        root.removeHandler(h)
        h.close()
    _INSTALLED.clear()
    root.setLevel(_apply_levels(os.environ.get("MESH_LOG", ""), level))
    for h in handlers:
        root.addHandler(h)
        _INSTALLED.append(h)
    return root


def init_production_logging(level: str = "info", log_dir: Optional[Path] = None, backup_days: int = 7) -> Path:
    """File (daily rotation) + console logging; returns the log file's path."""
    log_dir = Path(log_dir) if log_dir else _meshnet_home() / "logs"
    log_dir.mkdir(parents=True, exist_ok=True)
    path = log_dir / "agent.log"
    fh = logging.handlers.TimedRotatingFileHandler(path, when="midnight", backupCount=backup_days, encoding="utf-8")
    fh.setFormatter(logging.Formatter(FILE_FORMAT))
    ch = logging.StreamHandler(sys.stdout)
    ch.setFormatter(logging.Formatter(CONSOLE_FORMAT))
    _install([fh, ch], level)
    logging.getLogger("mesh").info("production logging initialised: dir=%s level=%s", log_dir, level)
    return path


def init_simple_logging(level: str = "info") -> None:
    ch = logging.StreamHandler(sys.stdout)
    ch.setFormatter(logging.Formatter(CONSOLE_FORMAT))
    _install([ch], level)
