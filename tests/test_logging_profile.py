"""Logging (rotating file, JSON lines) and the per-stage profiler."""
import json
import logging


def test_rotating_json_log(tmp_path):
    from swarmllm_b200.utils.logsetup import get_logger, setup_logging
    f = tmp_path / "s.log"
    setup_logging(0, str(f), json_format=True, max_bytes=2000, backups=2)
    log = get_logger("test")
    for i in range(100):
        log.info("message %d", i)
    log.debug("hidden at info level")
    lines = f.read_text().strip().splitlines()
    rec = json.loads(lines[-1])
    assert rec["msg"] == "message 99" and rec["level"] == "info" and rec["logger"] == "swarmllm_b200.test"
    assert (tmp_path / "s.log.1").exists() and (tmp_path / "s.log.2").exists()
    assert not (tmp_path / "s.log.3").exists()
    setup_logging(0)   # drop the file handler again
    logging.getLogger("swarmllm_b200").handlers[0].close()


def test_stage_profiler_accounts_named_stages():
    from swarmllm_b200.utils.tracing import StageProfiler
    p = StageProfiler(enabled=True, sync=False)
    for _ in range(3):
        with p.stage("attention"):
            pass
        with p.stage("ffn_down+norm"):
            pass
    assert p.counts == {"attention": 3, "ffn_down+norm": 3}
    assert "attention" in p.report()
    off = StageProfiler(enabled=False)
    with off.stage("x"):
        pass
    assert off.counts == {}


def test_logging_settings_from_toml(tmp_path):
    from swarmllm_b200.utils.config import load_logging_settings
    from swarmllm_b200.utils.logsetup import setup_logging
    p = tmp_path / "c.toml"
    p.write_text('[logging]\nlevel = "warn"\nformat = "json"\nfile = "%s"\n' % (tmp_path / "x.log"))
    lg = load_logging_settings(str(p))
    assert lg == {"level": "warn", "json": True, "file": str(tmp_path / "x.log")}
    log = setup_logging(0, lg["file"], lg["json"], level=lg["level"])
    assert log.level == logging.WARNING
    assert load_logging_settings(None) == {}
    setup_logging(0)
