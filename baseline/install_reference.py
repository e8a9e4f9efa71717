"""Install the unmodified reference (Piper Offload 0.2.5) under ``baseline/_ref``.

Usage: ``python baseline/install_reference.py [/path/to/piper-offload]``

The base recipe is ``pip install --no-index --no-build-isolation --find-links
/opt/wheelhouse --target baseline/_ref <reference>``. In this image it fails:
the reference builds with ``uv_build`` (absent from the wheelhouse) and
declares Python >= 3.14. So the recipe falls back to copying the package
source tree ``src/piper_offload`` unchanged into ``baseline/_ref/piper_offload``
(a plain file copy: no file is edited). ``baseline/reference.py`` imports it on
Python 3.12 with postponed annotations. ``baseline/_ref`` is git-ignored; it is
test and measurement infrastructure (the GPU parity target and the speed bar of
the reference's Triton kernels), never imported by ``piper_offload_b200``.
"""

from __future__ import annotations

import json
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEST = HERE / "_ref"


def main(ref: Path) -> int:
    src = ref / "src" / "piper_offload"
    if not src.is_dir():
        print(f"no reference package at {src}", file=sys.stderr)
        return 1
    record = {"reference": str(ref)}
    with tempfile.TemporaryDirectory() as tmp:  # the reference tree is read-only: build from a copy
        work = Path(tmp) / "ref"
        shutil.copytree(ref, work)
        pip = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                              "--no-deps", "--find-links", "/opt/wheelhouse", "--target", str(Path(tmp) / "t"),
                              str(work)], capture_output=True, text=True)
        record["pip_rc"] = pip.returncode
        record["pip_tail"] = (pip.stdout + pip.stderr).strip().splitlines()[-1:] if pip.returncode else []
    if DEST.exists():
        shutil.rmtree(DEST)
    DEST.mkdir(parents=True)
    shutil.copytree(src, DEST / "piper_offload", ignore=shutil.ignore_patterns("__pycache__"))
    for name in ("pyproject.toml", "LICENSE", "NOTICE"):
        if (ref / name).exists():
            shutil.copy2(ref / name, DEST / name)
    record["method"] = "pip" if record["pip_rc"] == 0 else "source copy of src/piper_offload (pip build failed)"
    (DEST / "INSTALL.json").write_text(json.dumps(record, indent=1))
    print(json.dumps(record))
    return 0


if __name__ == "__main__":
    sys.exit(main(Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")))
