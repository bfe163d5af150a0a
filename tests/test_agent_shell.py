"""Agent shell on CPU: error taxonomy, resource manager (allocation margin, lock cooldown,
persistence, re-pin after restart, HBM commitments), shard registry lifecycle and persistence
(also from two processes at once), model description from an on-disk model, rotating logs."""
import json
import logging
import logging.handlers
import multiprocessing as mp
import time

import pytest

from mesh_b200 import errors
from mesh_b200.models.registry import (ModelInfo, ShardRegistry, ShardStatus, assignment_by_columns,
                                       record_shard_load, shard_key)
from mesh_b200.runtime.resources import (ResourceManager, format_bytes, kv_pages_for,
                                         parse_memory_string)

GB = 10 ** 9


# ------------------------------------------------------------------------------------ errors
def test_error_categories_and_context():
    assert isinstance(errors.IoError("x"), OSError) and isinstance(errors.ConfigError("x"), ValueError)
    assert isinstance(errors.HttpError("x"), errors.NetworkError)
    e = errors.CooldownActive(5)
    assert e.remaining_hours == 5 and "5 hours" in str(e) and isinstance(e, errors.ResourceError)
    wrapped = errors.context("reading shard", FileNotFoundError("gone"))
    assert isinstance(wrapped, errors.IoError) and "reading shard: gone" in str(wrapped)
    assert isinstance(errors.context("x", KeyError("k")), errors.ExecutionError)
    assert type(errors.context("x", errors.QueueError("q"))) is errors.QueueError


# ---------------------------------------------------------------------------------- resources
@pytest.mark.parametrize("s,want", [("7GB", 7 * GB), ("7GiB", 7 << 30), ("512MB", 512 * 10 ** 6),
                                    ("1.5 GiB", int(1.5 * (1 << 30))), ("16G", 16 << 30), ("4096", 4096),
                                    ("2kib", 2048), ("3KB", 3000)])
def test_parse_memory_string(s, want):
    assert parse_memory_string(s) == want


@pytest.mark.parametrize("bad", ["", "GB", "-1GB", "seven", "1.5"])
def test_parse_memory_string_rejects(bad):
    with pytest.raises(errors.ConfigError):
        parse_memory_string(bad)


def test_format_bytes():
    assert format_bytes(999) == "999 bytes" and format_bytes(1500) == "1.5 KB"
    assert format_bytes(183 * GB) == "183.0 GB"


def test_host_lock_margin_cooldown_and_restart(tmp_path):
    cfg = tmp_path / "resource_lock.toml"
    rm = ResourceManager(cfg, pool="host", host_total=64 * GB, gpu_totals=[])
    with pytest.raises(errors.ResourceError):
        rm.set_allocation(63 * GB)  # the 7% margin does not fit
    with pytest.raises(errors.ResourceError):
        rm.lock()  # nothing allocated yet
    rm.set_allocation(1 << 20, cooldown_hours=24)  # 1 MiB: small enough to pin here
    assert rm.cfg.locked_memory == int((1 << 20) * 1.07)
    rm.lock()
    assert rm.is_locked and rm.is_pinned
    with pytest.raises(errors.ResourceError):
        rm.lock()
    with pytest.raises(errors.ResourceError):
        rm.set_allocation(2 << 20)
    with pytest.raises(errors.CooldownActive) as ei:
        rm.unlock()
    assert ei.value.remaining_hours == 24
    with pytest.raises(errors.CooldownActive) as ei:
        rm.unlock(now=time.time() + 23.5 * 3600)
    assert ei.value.remaining_hours == 1  # rounded up
    st = rm.status()
    assert st["locked"] and st["pinned"] and st["pool"] == "host"
    rm.close()
    # restart: the commitment is read back and re-pinned
    rm2 = ResourceManager(cfg, host_total=64 * GB, gpu_totals=[])
    assert rm2.is_locked and rm2.is_pinned and rm2.pool == "host" and rm2.cfg.user_allocated == 1 << 20
    rm2.unlock(now=time.time() + 24 * 3600 + 1)
    assert not rm2.is_locked and not rm2.is_pinned
    assert not ResourceManager(cfg, host_total=64 * GB, gpu_totals=[]).is_locked
    with pytest.raises(errors.ResourceError):
        rm2.unlock()


def test_hbm_commitment_checks_free_memory_and_sizes_kv(tmp_path):
    hbm = 183 * GB
    free = [170 * GB] * 8
    rm = ResourceManager(tmp_path / "r.toml", host_total=2000 * GB, gpu_totals=[hbm] * 8, gpu_free=lambda: free)
    assert rm.pool == "hbm" and rm.total_memory == hbm
    rm.set_allocation(150 * GB, cooldown_hours=0)
    rm.lock()
    assert rm.is_locked and not rm.is_pinned  # nothing pinned on the host for HBM
    rm.unlock()
    free[3] = 100 * GB
    with pytest.raises(errors.ResourceError, match=r"\[3\]"):
        rm.lock()
    # Llama-3-8B at TP1: 16 GB of weights; a 16-token page of K and V for 32 layers x 8 heads x 128
    page = 2 * 32 * 8 * 16 * 128 * 2
    assert kv_pages_for(150 * GB, 16 * GB, page) == (150 * GB - 16 * GB - (2 << 30)) // page
    with pytest.raises(errors.ResourceError):
        kv_pages_for(10 * GB, 16 * GB, page)


# --------------------------------------------------------------------------------- registry
def test_shard_lifecycle_and_persistence(tmp_path):
    reg = ShardRegistry(tmp_path)
    a = assignment_by_columns("llama3-8b", 1, 4, 4096)
    assert (a.column_start, a.column_end) == (1024, 2048)
    assert assignment_by_columns("m", 2, 3, 100).column_end == 100  # last takes the remainder
    s = reg.assign_shard(a)
    k = s.key
    assert k == shard_key("llama3-8b", 1, 4) and reg.status(k) == ShardStatus.PENDING
    assert s.contains_column(1024) and not s.contains_column(2048) and s.num_columns() == 1024
    with pytest.raises(errors.ConfigError):
        reg.mark_loaded(k, 10)  # not downloaded yet
    reg.update_download_progress(k, 0.5)
    assert reg.status(k) == ShardStatus.DOWNLOADING and reg.get_shard(k).download_progress == 0.5
    reg.mark_downloaded(k, tmp_path / "x.safetensors", "ab" * 32)
    reg.mark_loaded(k, 4 * GB, "cuda:1")
    assert reg.is_ready(k) and [x.key for x in reg.ready_shards()] == [k] and reg.total_memory_usage() == 4 * GB
    # a second process's view sees the same state
    again = ShardRegistry(tmp_path)
    got = again.get_shard(k)
    assert got.status == ShardStatus.READY and got.device == "cuda:1" and got.file_hash == "ab" * 32
    reg.mark_unloaded(k)
    assert reg.status(k) == ShardStatus.DOWNLOADED and reg.total_memory_usage() == 0
    reg.mark_error(k, "hash mismatch")
    assert ShardRegistry(tmp_path).get_shard(k).error == "hash mismatch"
    reg.remove_shard(k)
    assert ShardRegistry(tmp_path).get_shard(k) is None
    with pytest.raises(errors.ConfigError):
        reg.update_status(k, ShardStatus.READY)
    with pytest.raises(errors.ConfigError):
        reg.assign_shard(type(a)("m", 3, 2, 0, 8))  # position outside the group


def test_model_registration(tmp_path):
    reg = ShardRegistry(tmp_path)
    info = ModelInfo(model_id="llama3-70b", num_kv_heads=8, tensor_parallelism_dim=8192,
                     total_size_bytes=141 * GB, min_workers=2)
    reg.register_model(info)
    m = ShardRegistry(tmp_path).get_model("llama3-70b")
    assert m.total_size_bytes == 141 * GB and [x.model_id for x in reg.list_models()] == ["llama3-70b"]
    assert m.memory_for_workers(8) == 141 * GB // 8 + (141 * GB // 8) // 10
    assert m.memory_for_workers(0) == 141 * GB and m.columns_per_worker(8) == 1024
    assert m.can_run_with_workers(2) and not m.can_run_with_workers(1)
    assert m.valid_worker_counts() == [1, 2, 4, 8]


def _record(d, pos):
    reg = ShardRegistry(d)
    for i in range(20):
        a = assignment_by_columns(f"m{i % 2}", pos, 2, 64)
        k = reg.assign_shard(a).key
        reg.mark_downloaded(k, f"/p{pos}", "00")
        reg.mark_loaded(k, 100 + pos, f"cuda:{pos}")


def test_two_processes_record_their_own_shards(tmp_path):
    ps = [mp.get_context("spawn").Process(target=_record, args=(str(tmp_path), r)) for r in range(2)]
    [p.start() for p in ps]
    [p.join(60) for p in ps]
    assert all(p.exitcode == 0 for p in ps)
    reg = ShardRegistry(tmp_path)
    assert len(reg.ready_shards()) == 4  # two models x two positions, none lost to the other writer
    assert reg.total_memory_usage() == 2 * (100 + 101)


def test_model_info_from_disk_and_record_load(tmp_path):
    from mesh_b200.config import get_preset
    from mesh_b200.models.artifacts import assignment_for, load_shard, write_model
    from mesh_b200.models.weights import synthetic_reference_weights
    cfg = get_preset("tiny")
    out = write_model(tmp_path / "store", "tiny-m", synthetic_reference_weights(cfg, seed=3), 2)
    info = ModelInfo.from_model_dir(out, gpu_bytes=10 ** 12)
    assert info.model_id == "tiny-m" and info.num_layers == cfg.num_layers and info.min_workers == 1
    assert info.total_size_bytes == cfg.param_count() * 2 and len(info.shard_urls) == 2
    assert info.valid_worker_counts()[-1] == cfg.num_kv_heads
    with pytest.raises(errors.ResourceError):
        ModelInfo.from_model_dir(out, gpu_bytes=1000)
    reg = ShardRegistry(tmp_path / "reg")
    a = assignment_for(out, "tiny-m", 1, 2)
    load_shard(out, a)
    k = record_shard_load(reg, out, a, 12345, "cuda:1")
    man = json.loads((out / "shard-1-of-2.manifest.json").read_text())
    s = ShardRegistry(tmp_path / "reg").get_shard(k)
    assert s.status == ShardStatus.READY and s.file_hash == man["expected_sha256"] and s.memory_bytes == 12345


# ------------------------------------------------------------------------------------ logging
def test_production_logging_writes_file_and_honours_env(tmp_path, monkeypatch):
    from mesh_b200.utils.logs import init_production_logging, init_simple_logging
    monkeypatch.setenv("MESH_LOG", "mesh.noisy=error,debug")
    path = init_production_logging("info", tmp_path / "logs")
    assert logging.getLogger().level == logging.DEBUG
    logging.getLogger("mesh.test").debug("hello %d", 7)
    logging.getLogger("mesh.noisy").warning("suppressed")
    for h in logging.getLogger().handlers:
        h.flush()
    text = path.read_text()
    assert "mesh.test" in text and "hello 7" in text and "suppressed" not in text
    monkeypatch.delenv("MESH_LOG")
    init_simple_logging("warning")  # replaces the file handler
    assert logging.getLogger().level == logging.WARNING
    assert not any(isinstance(h, logging.handlers.TimedRotatingFileHandler) for h in logging.getLogger().handlers)
    logging.getLogger("mesh.noisy").setLevel(logging.NOTSET)
