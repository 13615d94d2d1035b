"""Extracts the released Flash model's `text_config` from the reference's
crates/core/fixtures/release/flash-config.json into flash_text_config.json
(the architecture only; the geometry test compares flash_config() with it).

    python tests/golden/make_flash_config.py <path to the reference project>
"""
import json
import sys
from pathlib import Path


def main(ref: str) -> None:
    src = Path(ref) / "crates" / "core" / "fixtures" / "release" / "flash-config.json"
    text = json.loads(src.read_text())["text_config"]
    out = Path(__file__).resolve().parent / "flash_text_config.json"
    out.write_text(json.dumps(text, indent=1, sort_keys=True) + "\n")
    print(f"wrote {out} from {src}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_flash_config.py <reference project root>")
    main(sys.argv[1])
