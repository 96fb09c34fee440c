"""Copies the reference's vendored parity fixtures into tests/golden/.

Source: tests/parity_test/out/fixtures/ of agkdc1/SPIRV_INFERENCE (raw
little-endian float32 vectors plus manifest.json with sha256 and the
thresholds of tests/parity_test/generate_fixtures.py:108-113).  Each file's
sha256 is checked against the reference manifest before it is copied.  As a
second check the reference generator script itself is run into a temporary
directory (it is pure Python with no dependencies) and its output must be
byte-identical to the vendored files.

Run from the repository root in a checkout that has the reference mounted:
    python tests/golden/make_golden.py /path/to/SPIRV_INFERENCE
"""
import hashlib
import os
import json
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    src = Path(ref_root) / "tests" / "parity_test" / "out" / "fixtures"
    manifest = json.loads((src / "manifest.json").read_text())
    with tempfile.TemporaryDirectory() as tmp:
        gen = Path(ref_root) / "tests" / "parity_test" / "generate_fixtures.py"
        subprocess.run([sys.executable, str(gen), "--out", tmp], check=True)
        for name, meta in manifest["files"].items():
            data = (src / meta["path"]).read_bytes()
            if hashlib.sha256(data).hexdigest() != meta["sha256"]:
                raise SystemExit(f"sha256 mismatch for vendored {name}")
            if (Path(tmp) / meta["path"]).read_bytes() != data:
                raise SystemExit(f"regenerated {name} differs from the vendored file")
            (HERE / meta["path"]).write_bytes(data)
    shutil.copy(src / "manifest.json", HERE / "manifest.json")
    print(f"copied {len(manifest['files'])} fixtures")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPX_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_golden.py <reference root> (or set SPX_REFERENCE_ROOT)")
    main(root)
