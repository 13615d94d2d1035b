"""Generates tests/golden/head_fixture.npz from the reference's own golden
fixture of the learned joint schema head (crates/core/fixtures/synthetic/
head.safetensors, head-input.safetensors and head-config.json of tyrchen/clef-rs).

The reference's test `head_parity` (crates/core/src/models/mod.rs:176-235)
runs `Head::forward` on `hidden` [20, 16] and `output_embeddings` [64, 16]
with ids 0..19 and three questions of kinds 0, 1, 2 (spans listed in
QUESTIONS below, copied from that test) and compares each question's logits
with `logits.{i}` within 1e-5 + 1e-4|e| (mod.rs:75-86). This script only
re-packages the tensors (names, shapes and values unchanged) into one .npz so
the tests run where the reference checkout is absent.

Usage: python tests/golden/make_head_golden.py REFERENCE_ROOT
"""
import json
import sys
from pathlib import Path

import numpy as np
from safetensors.numpy import load_file

# (kind, instruction span, option spans) of mod.rs:186-203, spans [start, end).
QUESTIONS = [
    (0, (1, 3), [(3, 5), (5, 7)]),
    (1, (7, 9), [(9, 11), (11, 13), (13, 15)]),
    (2, (15, 17), [(17, 18), (18, 19)]),
]


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} <checkout of the reference project>")
    root = Path(sys.argv[1])
    fx = root / "crates/core/fixtures/synthetic"
    weights = load_file(str(fx / "head.safetensors"))
    inputs = load_file(str(fx / "head-input.safetensors"))
    config = json.loads((fx / "head-config.json").read_text())
    out = {f"w:{k}": v.astype(np.float32) for k, v in weights.items()}
    out.update({f"in:{k}": v.astype(np.float32) for k, v in inputs.items()})
    out["ids"] = np.arange(20, dtype=np.int32)
    out["config_json"] = np.frombuffer(json.dumps(config).encode(), dtype=np.uint8)
    out["questions_json"] = np.frombuffer(json.dumps(QUESTIONS).encode(), dtype=np.uint8)
    dst = Path(__file__).with_name("head_fixture.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(weights)} weight tensors)")


if __name__ == "__main__":
    main()
