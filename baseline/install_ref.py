"""Install the unmodified reference (kvdlra) into ``baseline/_ref`` for the
benchmark's reference arm.

    python baseline/install_ref.py <reference checkout>

First tries the standard offline install
(``pip install --no-index --no-build-isolation --find-links /opt/wheelhouse
--target baseline/_ref <checkout>``).  The reference builds with hatchling,
which the offline wheelhouse does not carry, so when pip cannot build it this
places exactly the file set the reference's wheel contains -- the package
directory its ``pyproject.toml`` names under
``[tool.hatch.build.targets.wheel] packages`` (``src/kvdlra``) -- unmodified
into the target, as the wheel install would.  ``baseline/_ref`` is git-ignored:
nothing of the reference enters the repository's history.
"""

from __future__ import annotations

import shutil
import subprocess
import sys
import tomllib
from pathlib import Path

TARGET = Path(__file__).resolve().parent / "_ref"


def main() -> int:
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    src = Path(sys.argv[1]).resolve()
    meta = tomllib.loads((src / "pyproject.toml").read_text())
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
           "--no-deps", "--find-links", "/opt/wheelhouse", "--target", str(TARGET), str(src)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode == 0:
        print("installed with pip")
        return 0
    why = (res.stderr.strip().splitlines() or ["?"])[-1]
    print(f"pip could not build the reference ({why}); installing the wheel's file set")
    packages = meta["tool"]["hatch"]["build"]["targets"]["wheel"]["packages"]
    TARGET.mkdir(parents=True, exist_ok=True)
    for rel in packages:
        pkg = src / rel
        dest = TARGET / pkg.name
        if dest.exists():
            shutil.rmtree(dest)
        shutil.copytree(pkg, dest, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    (TARGET / "INSTALLED_FROM").write_text(f"{src} version {meta['project']['version']}\n")
    print(f"installed {', '.join(packages)} into {TARGET}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
