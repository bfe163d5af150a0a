"""Error taxonomy of the device agent (the categories of ``agent/src/errors.rs:1-60``).

Every error the agent raises on purpose derives from ``MeshError``; each category also derives
from the closest built-in exception, so callers that catch ``OSError`` / ``ValueError`` /
``RuntimeError`` keep working. ``context(msg)`` wraps any exception in a category with a message
prefix (the reference's ``ErrorContext``), chaining the original.
"""
from __future__ import annotations

import logging
from typing import Optional, Type

log = logging.getLogger("mesh.errors")


class MeshError(Exception):
    """Base of every error the agent raises on purpose."""
    category = "mesh"


class IoError(MeshError, OSError):
    category = "io"


class SerializationError(MeshError, ValueError):
    category = "serialization"


class CryptoError(MeshError, ValueError):
    category = "crypto"


class ConfigError(MeshError, ValueError):
    category = "config"


class NetworkError(MeshError, ConnectionError):
    category = "network"


class HttpError(NetworkError):
    category = "http"


class RegistrationError(MeshError, RuntimeError):
    category = "registration"


class ExecutionError(MeshError, RuntimeError):
    category = "execution"


class ResourceError(MeshError, RuntimeError):
    category = "resource"


class QueueError(MeshError, RuntimeError):
    category = "queue"


class CooldownActive(ResourceError):
    """An unlock asked for before the lock's cooldown has passed."""
    category = "cooldown_active"

    def __init__(self, remaining_hours: int):
        self.remaining_hours = int(remaining_hours)
        super().__init__(f"cooldown active: {self.remaining_hours} hours remaining until unlock")


_BY_BUILTIN = ((OSError, IoError), (ValueError, SerializationError))


def categorize(exc: BaseException) -> Type[MeshError]:
    """The category an arbitrary exception belongs to (``ExecutionError`` if none fits)."""
    if isinstance(exc, MeshError):
        return type(exc)
    for builtin, cat in _BY_BUILTIN:
        if isinstance(exc, builtin):
            return cat
    return ExecutionError


def context(msg: str, exc: BaseException, category: Optional[Type[MeshError]] = None) -> MeshError:
    """``category(f"{msg}: {exc}")`` chained to ``exc`` and logged at error level; use as
    ``raise context("loading shard", e) from e``."""
    cat = category or categorize(exc)
    if cat is CooldownActive:
        err = CooldownActive(getattr(exc, "remaining_hours", 0))
    else:
        err = cat(f"{msg}: {exc}")
    log.error("%s: %r", msg, exc)
    return err
