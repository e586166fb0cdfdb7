"""matrixman.config: keys, aliases, parsing, provenance and the lifecycle lock."""

import pytest

import importlib

config_module = importlib.import_module("matrixman_b200.config")
from matrixman_b200.config import Configuration


@pytest.fixture
def cfg(monkeypatch):
    for name in ("MATRIXMAN_SYNC_POLICY", "MATRIXMAN_ACTIVATION_POOL", "MATRIXMAN_TILE_LIMIT",
                 "MATRIXMAN_PROFILE", "MATRIXMAN_TRACE"):
        monkeypatch.delenv(name, raising=False)
    return Configuration()


def test_north_star_knobs_defaults(cfg):
    assert cfg.sync_policy == "safe"
    assert cfg.activation_pool == "safe"
    assert cfg.scratch_pool == "safe"
    assert cfg.tile_limit == 256
    assert cfg.resolved_tile_limit == 256


def test_aliases_and_camel_case(cfg):
    cfg.sync_policy = "relaxed"
    assert cfg.syncPolicy == "relaxed"
    cfg.activationPool = "deferred"
    assert cfg.activation_pool == "deferred"
    cfg.tile_limit = "auto"
    assert cfg.tileLimit == "auto" and cfg.resolvedTileLimit == 256
    assert cfg.source("sync_policy") == "python override"


def test_auto_sync_policy_resolves_to_relaxed(cfg):
    cfg.sync_policy = "auto"
    assert cfg.resolved_sync_policy == "relaxed"


def test_invalid_values_raise(cfg):
    with pytest.raises(ValueError):
        cfg.sync_policy = "sometimes"
    with pytest.raises(ValueError):
        cfg.scratch_pool = "eager"
    with pytest.raises(ValueError):
        cfg.tile_limit = 0
    with pytest.raises(AttributeError):
        cfg.not_a_setting = 1


def test_environment_precedence(monkeypatch):
    monkeypatch.setenv("MATRIXMAN_SYNC_POLICY", "relaxed")
    monkeypatch.setenv("MATRIXMAN_TILE_LIMIT", "128")
    c = Configuration()
    assert c.sync_policy == "relaxed" and c.tile_limit == 128
    assert c.source("tile_limit") == "environment"
    c.tile_limit = 64
    assert c.source("tile_limit") == "python override"
    c.reloadFromEnvironment()
    assert c.tile_limit == 128


def test_scratch_flag_compatibility(cfg):
    cfg.debug_fresh_scratch = True
    with pytest.raises(ValueError):
        cfg.scratch_epoch_pool = True
    assert cfg.scratch_policy == "fresh"


def test_lifecycle_lock(monkeypatch, cfg):
    from matrixman_b200 import runtime
    monkeypatch.setattr(runtime, "any_initialized", lambda: True)
    with pytest.raises(RuntimeError, match="must be set before backend initialization"):
        cfg.sync_policy = "relaxed"
    with pytest.raises(RuntimeError):
        cfg.activation_pool = "deferred"
    cfg.profile = "detail"  # not protected
    assert cfg.profile == "detail"
    assert config_module.config is not cfg  # module singleton untouched


def test_introspection(cfg, capsys):
    keys = cfg.keys()
    for k in ("sync_policy", "activation_pool", "scratch_pool", "tile_limit", "scratch_policy"):
        assert k in keys
    meta = cfg.metadata("sync_policy")
    assert meta["environment"] == "MATRIXMAN_SYNC_POLICY"
    assert meta["options"] == ("safe", "auto", "relaxed")
    assert meta["lifecycle"] == "set before backend initialization"
    text = cfg.describe("activation_pool")
    assert "deferred" in text
    assert cfg.show(as_text=True).startswith("MatrixMan configuration")
    assert dict(cfg.items())["tile_limit"] == 256
    with pytest.raises(ValueError):
        cfg.metadata("bogus")


def test_profile_and_trace_parsing(cfg):
    cfg.profile = True
    assert cfg.profile == "summary"
    cfg.profile = "0"
    assert cfg.profile is False
    cfg.trace = "detailed"
    assert cfg.trace == "detailed"


def test_module_level_profile_alias():
    import matrixman_b200 as matrixman
    old = matrixman.config._values["profile"]
    try:
        matrixman.profile = "detail"
        assert matrixman.profile == "detail"
        assert matrixman.config.profile == "detail"
    finally:
        matrixman.config._values["profile"] = old


def test_opengl_backend_rejected(cfg):
    with pytest.raises(ValueError):
        cfg.backend = "opengl"
