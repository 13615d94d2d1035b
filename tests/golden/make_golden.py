"""Generates tests/golden/backbone_fixture.npz from the reference's own golden
fixture (crates/core/fixtures/synthetic/backbone*.safetensors and
backbone-config.json of tyrchen/clef-rs).

The reference produced those files with transformers 5.10.2 / torch 2.11.0,
seed 7729 (fixtures/synthetic/provenance.json); its CPU backbone must reproduce
`hidden` for ids 0..19 within 1e-5 + 1e-4|e| (crates/core/src/models/mod.rs:75-111).
This script only re-packages the tensors (names, shapes and values unchanged)
into one .npz so the tests can run where the reference checkout is absent.

Usage: python tests/golden/make_golden.py REFERENCE_ROOT
"""
import json
import sys
from pathlib import Path

import numpy as np
from safetensors.numpy import load_file


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} <checkout of the reference project>")
    root = Path(sys.argv[1])
    fx = root / "crates/core/fixtures/synthetic"
    weights = load_file(str(fx / "backbone.safetensors"))
    expected = load_file(str(fx / "backbone-output.safetensors"))["hidden"]
    config = json.loads((fx / "backbone-config.json").read_text())
    out = {f"w:{k}": v.astype(np.float32) for k, v in weights.items()}
    out["expected_hidden"] = expected.astype(np.float32)
    out["ids"] = np.arange(20, dtype=np.int32)
    out["config_json"] = np.frombuffer(json.dumps(config).encode(), dtype=np.uint8)
    dst = Path(__file__).with_name("backbone_fixture.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(weights)} tensors)")


if __name__ == "__main__":
    main()
