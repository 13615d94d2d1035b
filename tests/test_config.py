"""Model geometry: the Flash geometry the engine benchmarks and parity-tests
(`flash_config`) is the released model's architecture, read from its
`text_config` (crates/core/fixtures/release/flash-config.json, extracted by
tests/golden/make_flash_config.py) the way Backbone::load reads it
(crates/core/src/models/qwen.rs:193-277)."""
import json
from pathlib import Path

from clef_b200.config import benchmark_config, flash_config, from_text_config

ROOT = Path(__file__).resolve().parents[1]


def released_text_config() -> dict:
    return json.loads((ROOT / "tests" / "golden" / "flash_text_config.json").read_text())


def test_flash_config_is_the_released_architecture():
    released = from_text_config(released_text_config(), head_outputs=7).describe()
    assert flash_config(layers=32, head_outputs=7).describe() == released


def test_benchmark_config_differs_from_flash_only_in_width():
    flash = flash_config().describe()
    bench = benchmark_config().describe()
    differing = {k for k in flash if flash[k] != bench[k]}
    assert differing == {"hidden_size", "intermediate_size"}
    assert (bench["hidden_size"], bench["intermediate_size"]) == (2560, 9216)
